"""FP32 prefill and chunked-prefill kernels vs the oracle (kernel/attention.c:252-381,
:413-543 semantics), through attention_prefill_gqa / attention_chunked_prefill_gqa."""

import ctypes

import numpy as np
import pytest
import torch

from gpu_helpers import (TOL_BF16_MAX, TOL_BF16_REL, TOL_MAX, TOL_REL, bf16_round, check, dev, fill_layer,
                         head_first, new_cache, vp)
from oracle import max_abs, rel_l2

pytestmark = pytest.mark.gpu
SCALE = ctypes.c_float(0.08838834764831843)


def _prefill(pkg, lib, q, k, v, Sk, mode, scratch=None):
    Sq = q.shape[0]
    if mode == "device":
        qd, kd, vd = dev(q), dev(k), dev(v)
        od = torch.zeros_like(qd)
        lib.attention_prefill_gqa(vp(qd), vp(kd), vp(vd), vp(od), Sq, Sk, SCALE, None, None, None, None)
        assert lib.attn_sync() == 0, pkg.last_error(lib)
        check(pkg, lib, "prefill")
        return od.cpu().numpy()
    out = np.zeros_like(q)
    hm = [None] * 4
    if scratch is not None:
        s = ctypes.cast(scratch, ctypes.POINTER(ctypes.c_void_p * 14)).contents
        hm = [s[8], s[9], s[10], s[11]]  # q_hm, k_hm, v_hm, o_hm (kernel/scratch.h:27-30)
    lib.attention_prefill_gqa(vp(q), vp(k), vp(v), vp(out), Sq, Sk, SCALE, *hm)
    check(pkg, lib, "prefill")
    return out


def test_golden_prefill(pkg, lib, golden):
    g = golden("prefill_s36.npz")
    S = g["q"].shape[0]
    for mode in ("host", "device"):
        out = _prefill(pkg, lib, g["q"], g["k"], g["v"], S, mode)
        assert max_abs(out, g["out"]) <= TOL_MAX and rel_l2(out, g["out"]) <= TOL_REL, mode


def test_prefill_through_scratch_staging(pkg, lib, golden):
    g = golden("prefill_s36.npz")
    s = lib.decoder_scratch_alloc(64)
    assert s, pkg.last_error(lib)
    try:
        out = _prefill(pkg, lib, g["q"], g["k"], g["v"], g["q"].shape[0], "host", scratch=s)
    finally:
        lib.decoder_scratch_free(s)
    assert max_abs(out, g["out"]) <= TOL_MAX and rel_l2(out, g["out"]) <= TOL_REL


@pytest.mark.parametrize("S", [1024, 1500, 4096])
def test_prefill_host_pipelined_matches_device(pkg, lib, S):
    """Host q/k/v/output with every query seeing its own key (Sk = Sq >= 1024) take the pipelined
    path: rows go in by chunks of whole query tiles while earlier chunks are split and attended,
    and each chunk's output comes back on its own stream.  The chunks compute the same query tiles
    over the same hi/lo K/V rows as one launch over device buffers, so the results are equal bit
    for bit -- from pageable numpy buffers, and from page-locked buffers through the scratch's
    device slots twice in a row (the second call reuses the staging the first one left)."""
    rng = np.random.default_rng(S)
    q = rng.standard_normal((S, 16, 128), dtype=np.float32)
    k = rng.standard_normal((S, 8, 128), dtype=np.float32)
    v = rng.standard_normal((S, 8, 128), dtype=np.float32)
    want = _prefill(pkg, lib, q, k, v, S, "device")
    np.testing.assert_array_equal(_prefill(pkg, lib, q, k, v, S, "host"), want)
    s = lib.decoder_scratch_alloc(S)
    assert s, pkg.last_error(lib)
    try:
        slots = ctypes.cast(s, ctypes.POINTER(ctypes.c_void_p * 14)).contents
        hm = [slots[8], slots[9], slots[10], slots[11]]
        qp, kp, vpin = (torch.from_numpy(x).pin_memory() for x in (q, k, v))
        outp = torch.zeros((S, 16, 128), dtype=torch.float32).pin_memory()
        for _ in range(2):
            outp.fill_(0.0)
            lib.attention_prefill_gqa(vp(qp), vp(kp), vp(vpin), vp(outp), S, S, SCALE, *hm)
            check(pkg, lib, "prefill (page-locked)")
            np.testing.assert_array_equal(outp.numpy(), want)
    finally:
        lib.decoder_scratch_free(s)


@pytest.mark.parametrize("S,Sk", [(1, 1), (2, 2), (31, 31), (32, 32), (33, 33), (64, 64), (65, 65), (100, 100),
                                  (257, 257), (1024, 1024), (40, 20), (50, 80)])
def test_prefill_vs_oracle(pkg, lib, oracle, S, Sk):
    rng = np.random.default_rng(S * 31 + Sk)
    n = max(S, Sk)
    q = rng.standard_normal((S, 16, 128), dtype=np.float32)
    k = rng.standard_normal((n, 8, 128), dtype=np.float32)
    v = rng.standard_normal((n, 8, 128), dtype=np.float32)
    want = oracle.prefill(q, k, v, Sk)
    out = _prefill(pkg, lib, q, k, v, Sk, "device" if S % 2 else "host")
    assert max_abs(out, want) <= TOL_MAX and rel_l2(out, want) <= TOL_REL


def test_config1_prefill_chain(pkg, lib, oracle):
    """Config 1: raw Q/K through QK-RMSNorm + M-RoPE (oracle, as decoder.c does on the
    host), then the CUDA prefill, against the oracle prefill."""
    import importlib
    wl = importlib.import_module(pkg.__name__ + ".workloads")
    c = wl.config1(seed=0, n_decode=0)
    cos, sin = oracle.mrope_cos_sin_3d(c["pos"])
    q, k = oracle.qk_norm_rope(c["q"], c["k"], c["q_norm"], c["k_norm"], cos, sin)
    want = oracle.prefill(q, k, c["v"])
    out = _prefill(pkg, lib, q, k, c["v"], q.shape[0], "host")
    assert max_abs(out, want) <= TOL_MAX and rel_l2(out, want) <= TOL_REL


def test_golden_chunked(pkg, lib, golden):
    g = golden("chunked_c20_off37.npz")
    n = g["k_rows"].shape[0]
    off = int(g["pos_offset"])
    h = new_cache(pkg, lib, n + 3, pkg.ATTN_KV_F32)
    try:
        fill_layer(pkg, lib, h, 9, g["k_rows"], g["v_rows"])
        out = np.zeros_like(g["q"])
        lib.attention_chunked_prefill_gqa(vp(g["q"]), h, vp(out), 9, g["q"].shape[0], off, SCALE)
        check(pkg, lib, "chunked")
    finally:
        lib.kv_cache_free(h)
    assert max_abs(out, g["out"]) <= TOL_MAX and rel_l2(out, g["out"]) <= TOL_REL


@pytest.mark.parametrize("chunk,off", [(1, 0), (1, 511), (32, 0), (33, 256), (70, 31), (512, 1536)])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_chunked_vs_oracle(pkg, lib, oracle, chunk, off, dtype):
    rng = np.random.default_rng(chunk * 1009 + off)
    n = off + chunk
    q = rng.standard_normal((chunk, 16, 128), dtype=np.float32)
    k = rng.standard_normal((n, 8, 128), dtype=np.float32)
    v = rng.standard_normal((n, 8, 128), dtype=np.float32)
    kv_dt = pkg.ATTN_KV_F32 if dtype == "f32" else pkg.ATTN_KV_BF16
    h = new_cache(pkg, lib, n, kv_dt)
    try:
        fill_layer(pkg, lib, h, 0, k, v)
        qd = dev(q)
        od = torch.zeros_like(qd)
        lib.attention_chunked_prefill_gqa(vp(qd), h, vp(od), 0, chunk, off, SCALE)
        assert lib.attn_sync() == 0, pkg.last_error(lib)
        out = od.cpu().numpy()
    finally:
        lib.kv_cache_free(h)
    if dtype == "bf16":
        exact = oracle.chunked_prefill(q, head_first(bf16_round(k)), head_first(bf16_round(v)), off)
        assert max_abs(out, exact) <= TOL_MAX and rel_l2(out, exact) <= TOL_REL
        ref32 = oracle.chunked_prefill(q, head_first(k), head_first(v), off)
        assert max_abs(out, ref32) <= TOL_BF16_MAX and rel_l2(out, ref32) <= TOL_BF16_REL
    else:
        want = oracle.chunked_prefill(q, head_first(k), head_first(v), off)
        assert max_abs(out, want) <= TOL_MAX and rel_l2(out, want) <= TOL_REL


def test_prefill_rejects_bad_arguments(pkg, lib):
    q = np.zeros((4, 16, 128), dtype=np.float32)
    lib.attn_clear_error()
    lib.attention_prefill_gqa(vp(q), None, vp(q), vp(q), 4, 4, SCALE, None, None, None, None)
    assert "NULL" in pkg.last_error(lib)
    lib.attn_clear_error()
    lib.attention_prefill_gqa(vp(q), vp(q), vp(q), vp(q), -1, 4, SCALE, None, None, None, None)
    assert pkg.last_error(lib)
    lib.attn_clear_error()
    h = new_cache(pkg, lib, 8, pkg.ATTN_KV_F32)
    try:
        lib.attention_chunked_prefill_gqa(vp(q), h, vp(q), 0, 4, 6, SCALE)  # rows 6..9 > max_seq 8
        assert "exceed" in pkg.last_error(lib)
    finally:
        lib.attn_clear_error()
        lib.kv_cache_free(h)
