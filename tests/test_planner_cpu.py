"""Split planning of the decode kernels (host logic, no GPU): tyb_decode_plan decides which decode
kernel a call runs and how the rows are divided among CTAs.  Without a device the library plans for
148 SMs (a B200).  The invariants checked here are the ones the kernels and the workspaces rely on:
every split (span) is non-empty and together they cover the sequence; the tensor-core form's tiles
fit its 256-row TMA boxes and its launch is one wave at one CTA per SM; the streaming form's spans
are whole 96-row stages and fit one wave at two CTAs per SM; every plan fits the per-cache record
workspace (sized for 16-row splits) and, for the no-allocation entry point, its fixed scratch."""

import ctypes

import pytest

import gpu_helpers  # noqa: F401  (puts the package on sys.path)
from gpu_helpers import load_pkg_and_lib

SMS = 148
KV_HEADS = 8


@pytest.fixture(scope="module")
def lib():
    _, lib = load_pkg_and_lib()
    return lib


def plan(lib, kv_len, dtype, batch=1):
    c, n = ctypes.c_int(), ctypes.c_int()
    lib.tyb_decode_plan(batch, kv_len, dtype, ctypes.byref(c), ctypes.byref(n))
    return c.value, n.value


LENGTHS = sorted({1, 2, 15, 16, 17, 95, 96, 97, 100, 255, 256, 257, 1024, 2047, 4095, 4096, 4097, 4352,
                  4600, 4607, 4608, 4609, 4610, 6000, 8192, 12289, 20001, 24576, 32768, 32769, 33792, 65536,
                  131072, 262144})


@pytest.mark.parametrize("kv_len", LENGTHS)
def test_bf16_single_sequence_plan(lib, kv_len):
    chunk, nsplit = plan(lib, kv_len, 1)
    assert chunk > 0 and nsplit > 0
    assert chunk * nsplit >= kv_len and (nsplit - 1) * chunk < kv_len  # covered, no empty split
    one_wave = -(-kv_len // 256) * KV_HEADS <= SMS
    if one_wave:  # tensor-core form: 16-row tiles, one TMA box per half, one CTA per SM
        assert chunk % 16 == 0 and chunk <= 256
        assert nsplit * KV_HEADS <= SMS
    else:  # streaming form: whole 96-row stages, one wave at two CTAs per SM
        assert chunk % 96 == 0
        assert nsplit * KV_HEADS <= 2 * SMS
    # the per-cache record workspace holds max_seq/16 + 1 splits per KV head (max_seq >= kv_len)
    assert nsplit <= (kv_len + 15) // 16 + 1


@pytest.mark.parametrize("kv_len", LENGTHS)
def test_f32_single_sequence_plan(lib, kv_len):
    chunk, nsplit = plan(lib, kv_len, 0)
    assert chunk > 0 and nsplit > 0
    assert chunk * nsplit >= kv_len and (nsplit - 1) * chunk < kv_len
    assert chunk % 16 == 0
    assert nsplit <= (kv_len + 15) // 16 + 1
    if kv_len <= 24576:  # the no-allocation entry point's fixed scratch holds 256 splits
        assert nsplit <= 256


@pytest.mark.parametrize("batch", [2, 8, 64])
@pytest.mark.parametrize("dtype", [0, 1])
def test_request_batch_plan_covers_longest(lib, batch, dtype):
    for kv_len in (1, 1024, 4097, 8192):
        chunk, nsplit = plan(lib, kv_len, dtype, batch)
        assert chunk * nsplit >= kv_len and (nsplit - 1) * chunk < kv_len
        assert nsplit <= (kv_len + 15) // 16 + 1
