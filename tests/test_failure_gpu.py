"""Failure detection, exercised without faulting the GPU:

* a bounded wait that runs out: the output gather of a two-rank decode whose second rank (a
  child process on the same GPU that allocates its exchange buffer and then launches nothing)
  never raises its flag.  With the wait limit at 1 ms the gather's wait kernel gives up, the
  call reports "wait timed out" through attn_last_error(), and the next plain call on the same
  context succeeds and matches the unsharded decode;
* allocation failures, injected on the host (TYB_FAULT_ALLOC): kv_cache_alloc_ex and
  decoder_scratch_alloc return NULL with everything they had allocated freed, as the reference's
  allocators do (kernel/kv_cache.c:17-30, kernel/scratch.c:58-64);
* attn_workspace_reserve: calls within the reserved sizes allocate no device memory.
"""

import ctypes
import os

import numpy as np
import pytest
import torch

from gpu_helpers import fill_layer, new_cache, vp

pytestmark = pytest.mark.gpu
SCALE = ctypes.c_float(0.08838834764831843)


def _silent_rank(conn, done):
    """Rank 1 of two: exchange buffer and IPC handle, then nothing until told to exit."""
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from gpu_helpers import load_pkg_and_lib
    torch.cuda.set_device(0)
    pkg, lib = load_pkg_and_lib()
    h = (ctypes.c_char * 64)()
    ok = lib.attn_gather_init(1, 2) == 0 and lib.attn_gather_handle(h) == 0
    conn.send(bytes(h) if ok else b"")
    done.wait(120)
    lib.attn_gather_close()


def test_gather_wait_runs_out_and_context_survives(pkg, lib):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    parent, child = ctx.Pipe()
    done = ctx.Event()
    p = ctx.Process(target=_silent_rank, args=(child, done))
    p.start()
    rng = np.random.default_rng(5)
    n = 3000
    k = rng.standard_normal((n + 2, 8, 128), dtype=np.float32)
    v = rng.standard_normal((n + 2, 8, 128), dtype=np.float32)
    h = new_cache(pkg, lib, n + 2, pkg.ATTN_KV_BF16)
    connected = False
    try:
        other = parent.recv()
        assert len(other) == 64, "rank 1 could not set up its exchange buffer"
        mine = (ctypes.c_char * 64)()
        assert lib.attn_gather_init(0, 2) == 0
        assert lib.attn_gather_handle(mine) == 0
        handles = (ctypes.c_char * 128).from_buffer_copy(bytes(mine) + other)
        assert lib.attn_gather_connect(handles) == 0, pkg.last_error(lib)
        connected = True
        fill_layer(pkg, lib, h, 2, k[:n], v[:n])
        pkg.cache_struct(h).seq_len = n
        q = torch.tensor(rng.standard_normal((16, 128), dtype=np.float32), device="cuda")
        kn, vn = torch.tensor(k[n], device="cuda"), torch.tensor(v[n], device="cuda")
        out = torch.zeros((16, 128), device="cuda")
        assert lib.attn_set_wait_limit_ns(1_000_000) == 0, pkg.last_error(lib)  # 1 ms
        lib.attn_clear_error()
        # rank 0 owns KV heads 0-3; rank 1's flag never rises
        assert lib.attention_decode_append_gqa_gathered(vp(q), vp(kn), vp(vn), h, vp(out), 2, SCALE, 0, 4) == 0
        assert lib.attn_sync() != 0
        assert "wait timed out" in pkg.last_error(lib)
        lib.attn_clear_error()
        assert lib.attn_set_wait_limit_ns(2_000_000_000) == 0
        lib.attn_gather_close()
        connected = False
        # the context is usable: a plain decode step runs and matches a second cache's
        want = torch.zeros((16, 128), device="cuda")
        h2 = new_cache(pkg, lib, n + 2, pkg.ATTN_KV_BF16)
        try:
            fill_layer(pkg, lib, h2, 2, k[:n], v[:n])
            pkg.cache_struct(h2).seq_len = n
            got = torch.full((16, 128), float("nan"), device="cuda")
            assert lib.attention_decode_append_gqa(vp(q), vp(kn), vp(vn), h, vp(got), 2, SCALE) == 0
            assert lib.attention_decode_append_gqa(vp(q), vp(kn), vp(vn), h2, vp(want), 2, SCALE) == 0
            assert lib.attn_sync() == 0, pkg.last_error(lib)
            assert torch.isfinite(got).all() and torch.equal(got, want)
        finally:
            lib.kv_cache_free(h2)
    finally:
        lib.attn_set_wait_limit_ns(2_000_000_000)
        if connected:
            lib.attn_gather_close()
        lib.kv_cache_free(h)
        done.set()
        p.join(60)


def _free_bytes():
    torch.cuda.synchronize()
    return torch.cuda.mem_get_info()[0]


@pytest.mark.parametrize("kv_dtype", [0, 1])
def test_cache_alloc_failure_frees_partial_state(pkg, lib, kv_dtype):
    lib.attn_clear_error()
    warm = lib.kv_cache_alloc_ex(64, kv_dtype)  # first-use set-up (status mirror) out of the way
    assert warm, pkg.last_error(lib)
    lib.kv_cache_free(warm)
    base = _free_bytes()
    try:
        for n in range(1, 7):  # each of its six device allocations in turn
            os.environ["TYB_FAULT_ALLOC"] = f"{n}:cache{kv_dtype}"
            assert not lib.kv_cache_alloc_ex(4096, kv_dtype), n
            msg = pkg.last_error(lib)
            assert "injected" in msg and "kv_cache_alloc" in msg, msg
            lib.attn_clear_error()
            assert abs(_free_bytes() - base) < (8 << 20), f"allocation {n} failed but memory stayed allocated"
        os.environ["TYB_FAULT_ALLOC"] = f"7:cache{kv_dtype}"  # past the last one: succeeds
        h = lib.kv_cache_alloc_ex(4096, kv_dtype)
        assert h, pkg.last_error(lib)
        lib.kv_cache_free(h)
    finally:
        os.environ.pop("TYB_FAULT_ALLOC", None)
    assert abs(_free_bytes() - base) < (8 << 20)


def test_scratch_alloc_failure_frees_partial_state(pkg, lib):
    lib.attn_clear_error()
    base = _free_bytes()
    try:
        for n in range(1, 13):  # 8 page-locked host buffers, then the 4 device slots
            os.environ["TYB_FAULT_ALLOC"] = f"{n}:scratch"
            assert not lib.decoder_scratch_alloc(2048), n
            assert "injected" in pkg.last_error(lib)
            lib.attn_clear_error()
            assert abs(_free_bytes() - base) < (8 << 20), f"allocation {n} failed but device memory stayed"
        os.environ["TYB_FAULT_ALLOC"] = "13:scratch"
        s = lib.decoder_scratch_alloc(2048)
        assert s, pkg.last_error(lib)
        lib.decoder_scratch_free(s)
    finally:
        os.environ.pop("TYB_FAULT_ALLOC", None)


def test_reserved_workspace_is_not_reallocated(pkg, lib, oracle):
    S = 640
    assert lib.attn_workspace_reserve(S, 4, 2048) == 0, pkg.last_error(lib)
    rng = np.random.default_rng(8)
    q = rng.standard_normal((S, 16, 128), dtype=np.float32)
    k = rng.standard_normal((S, 8, 128), dtype=np.float32)
    v = rng.standard_normal((S, 8, 128), dtype=np.float32)
    out = np.zeros_like(q)
    # first launches load their kernels' modules (device memory of their own): done before measuring
    lib.attention_prefill_gqa(vp(q[:16]), vp(k[:16]), vp(v[:16]), vp(out[:16]), 16, 16, SCALE, None, None, None,
                              None)
    pkg.check(lib, "warm-up")
    base = _free_bytes()
    lib.attention_prefill_gqa(vp(q), vp(k), vp(v), vp(out), S, S, SCALE, None, None, None, None)  # host buffers
    pkg.check(lib, "prefill")
    assert _free_bytes() == base, "a call within the reserved sizes allocated device memory"
    want = oracle.prefill(q, k, v)
    assert np.max(np.abs(out - want)) <= 2e-3
