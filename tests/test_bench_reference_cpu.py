"""The reference arm of bench.py on the host cores (no GPU): its JSON line keeps the bench contract,
ranks other than 0 stay silent under torchrun, and the OpenMP thread count it reports is the one
it runs with (torchrun exports OMP_NUM_THREADS=1 to its workers; the arm overrides it)."""

import ctypes
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "oracle"))
import oracle as orc  # noqa: E402


def _have_cpu_reference():
    return orc.RefLib.available() or Path(orc.ORACLE_LIB).exists()


def _run_arm(extra_env):
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "LOCAL_RANK", "WORLD_SIZE")}
    env.update(extra_env)
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "2",
                           "--warmup", "3"], capture_output=True, text=True, env=env, timeout=600, cwd=str(ROOT))


@pytest.mark.skipif(not _have_cpu_reference(), reason="oracle libraries not built (run __graft_entry__.build())")
def test_reference_arm_json_line():
    r = _run_arm({"OMP_NUM_THREADS": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["unit"] == "us/step" and d["higher_is_better"] is False
    assert d["value"] > 0 and d["steps"] == 2 and d["warmup"] == 3
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port")
    assert cb["value"] == d["value"]
    # the count reported is the count used: every core of the process's affinity
    assert cb["cores"] == orc.host_threads()
    assert d["e2e"]["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0


def test_reference_arm_other_ranks_do_nothing():
    r = _run_arm({"RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [ln for ln in r.stdout.splitlines() if ln.startswith("{")]


def test_set_host_threads_overrides_omp_env():
    try:
        gomp = ctypes.CDLL("libgomp.so.1")
    except OSError:
        pytest.skip("libgomp.so.1 not loadable")
    gomp.omp_get_max_threads.restype = ctypes.c_int
    before = gomp.omp_get_max_threads()
    try:
        assert orc.set_host_threads(2) == 2
        assert gomp.omp_get_max_threads() == 2
    finally:
        gomp.omp_set_num_threads(before)
    assert orc.host_threads() >= 1
