"""Tensor-core prefill (tcgen05/TMEM, BF16 operands, FP32 accumulation) with QK-RMSNorm and
M-RoPE fused, through attention_prefill_fused_gqa, against the oracle running the same chain
(kernel/decoder.c:73-117: RMSNorm, M-RoPE, append, attention).

Tolerances of the BF16 path (written here), about twice the largest errors measured on a B200
over these tests: against the oracle fed the same BF16-rounded normalised q, k and v, max-abs
TOL_TC_MAX and rel-L2 TOL_TC_REL (measured at most 1.9e-3 / 1.3e-3 with FP32 output) -- what remains
is the BF16 rounding of the softmax weights P before the P.V product and the order of FP32 sums --
plus TOL_OUT_BF16_* when the output is rounded to BF16 too (measured at most 5.1e-3 / 2.0e-3 in all);
against the unrounded FP32 chain, TOL_TC32_* (measured at most 7.5e-3 / 2.9e-3 with FP32 output,
4.4e-3 / 3.0e-3 for config 3 with BF16 inputs and output).
"""

import ctypes
import importlib

import numpy as np
import pytest
import torch

from gpu_helpers import bf16_round, d2h, dev, head_first, new_cache, vp
from oracle import max_abs, rel_l2

pytestmark = pytest.mark.gpu
SCALE = ctypes.c_float(0.08838834764831843)
EPS = ctypes.c_float(1e-6)
TOL_TC_MAX, TOL_TC_REL = 4e-3, 2.6e-3
TOL_OUT_BF16_MAX, TOL_OUT_BF16_REL = 6e-3, 1.6e-3
TOL_TC32_MAX, TOL_TC32_REL = 1.5e-2, 6e-3


def _inputs(pkg, S, seed, grid=None):
    wl = importlib.import_module(pkg.__name__ + ".workloads")
    rng = np.random.default_rng(seed)
    if grid:
        pos = wl.mrope_positions(*grid)
    else:
        n_vis = min(S, 24)
        gh = max(1, int(np.sqrt(n_vis)))
        pos = wl.mrope_positions(gh, n_vis // gh, S - (n_vis // gh) * gh)
    assert pos.shape[1] == S
    q, k, v = wl.qkv(rng, S)
    qn, kn = wl.norm_weights(rng)
    return q, k, v, qn, kn, pos


def _fused(pkg, lib, h, layer, q, k, v, qn, kn, cos, sin, in_bf16, out_bf16):
    tdt = torch.bfloat16 if in_bf16 else torch.float32
    qd, kd, vd = (torch.from_numpy(x).to(tdt).cuda() for x in (q, k, v))
    qnd, knd, cd, sd = dev(qn), dev(kn), dev(cos), dev(sin)
    od = torch.zeros(q.shape, dtype=torch.bfloat16 if out_bf16 else torch.float32, device="cuda")
    rc = lib.attention_prefill_fused_gqa(vp(qd), vp(kd), vp(vd), int(in_bf16), vp(qnd), vp(knd), vp(cd), vp(sd), h,
                                         layer, vp(od), int(out_bf16), q.shape[0], SCALE, EPS)
    assert rc == 0, pkg.last_error(lib)
    assert lib.attn_sync() == 0, pkg.last_error(lib)
    return od.float().cpu().numpy()


def _expect(oracle, q, k, v, qn, kn, cos, sin, in_bf16):
    if in_bf16:
        q, k, v = bf16_round(q), bf16_round(k), bf16_round(v)
    qr, kr = oracle.qk_norm_rope(q, k, qn, kn, cos, sin)
    exact = oracle.prefill(bf16_round(qr), bf16_round(kr), bf16_round(v))
    fp32 = oracle.prefill(qr, kr, v)
    return exact, fp32, kr


@pytest.mark.parametrize("S", [5, 130])
def test_fused_prefill_small(pkg, lib, oracle, S):
    q, k, v, qn, kn, pos = _inputs(pkg, S, 40 + S)
    cos, sin = oracle.mrope_cos_sin_3d(pos)
    h = new_cache(pkg, lib, S + 4, pkg.ATTN_KV_BF16)
    try:
        out = _fused(pkg, lib, h, 3, q, k, v, qn, kn, cos, sin, in_bf16=False, out_bf16=False)
        rows = d2h(lib.kv_cache_k(h, 3, 0), (8, S + 4, 128), np.uint16)[:, :S]
    finally:
        lib.kv_cache_free(h)
    exact, fp32, kr = _expect(oracle, q, k, v, qn, kn, cos, sin, False)
    print(f"S={S}: vs rounded max {max_abs(out, exact):.3e} rel {rel_l2(out, exact):.3e}; "
          f"vs fp32 max {max_abs(out, fp32):.3e} rel {rel_l2(out, fp32):.3e}")
    # The cache holds the normalised, rotated K in BF16 (one rounding; at most one ulp apart
    # from rounding the oracle's FP32 value, since RMSNorm's rsqrt differs in the last bits).
    got_k = (rows.astype(np.uint32) << 16).view(np.float32)
    want_k = head_first(bf16_round(kr))
    assert np.max(np.abs(got_k - want_k) / (np.abs(want_k) + 1e-3)) < 1.6e-2
    assert max_abs(out, exact) <= TOL_TC_MAX and rel_l2(out, exact) <= TOL_TC_REL
    assert max_abs(out, fp32) <= TOL_TC32_MAX and rel_l2(out, fp32) <= TOL_TC32_REL


@pytest.mark.parametrize("S", [1, 127, 128, 129, 256, 511, 1024])
@pytest.mark.parametrize("in_bf16,out_bf16", [(False, False), (True, True), (False, True)])
def test_fused_prefill_sizes(pkg, lib, oracle, S, in_bf16, out_bf16):
    q, k, v, qn, kn, pos = _inputs(pkg, S, 1000 + S)
    cos, sin = oracle.mrope_cos_sin_3d(pos)
    h = new_cache(pkg, lib, S, pkg.ATTN_KV_BF16)
    try:
        out = _fused(pkg, lib, h, 27, q, k, v, qn, kn, cos, sin, in_bf16, out_bf16)
    finally:
        lib.kv_cache_free(h)
    exact, fp32, _ = _expect(oracle, q, k, v, qn, kn, cos, sin, in_bf16)
    print(f"S={S} in_bf16={in_bf16} out_bf16={out_bf16}: vs rounded max {max_abs(out, exact):.3e} "
          f"rel {rel_l2(out, exact):.3e}; vs fp32 max {max_abs(out, fp32):.3e} rel {rel_l2(out, fp32):.3e}")
    tol_max = TOL_TC_MAX + (TOL_OUT_BF16_MAX if out_bf16 else 0.0)  # one more BF16 rounding of the output
    tol_rel = TOL_TC_REL + (TOL_OUT_BF16_REL if out_bf16 else 0.0)
    assert max_abs(out, exact) <= tol_max and rel_l2(out, exact) <= tol_rel


@pytest.mark.parametrize("off,S", [(1, 1), (100, 30), (128, 128), (300, 200), (1000, 129)])
def test_fused_prefill_chunked(pkg, lib, oracle, off, S):
    """A filled cache (rows [0, off)) plus S new tokens at positions off..off+S-1."""
    q, k, v, qn, kn, pos = _inputs(pkg, S, 7 * off + S)
    cos, sin = oracle.mrope_cos_sin_3d(pos)
    rng = np.random.default_rng(off)
    k_old = rng.standard_normal((off, 8, 128), dtype=np.float32)
    v_old = rng.standard_normal((off, 8, 128), dtype=np.float32)
    h = new_cache(pkg, lib, off + S + 3, pkg.ATTN_KV_BF16)
    try:
        lib.kv_cache_append_prefill(h, 9, vp(k_old), vp(v_old), off)
        pkg.check(lib, "fill")
        pkg.cache_struct(h).seq_len = off
        out = _fused(pkg, lib, h, 9, q, k, v, qn, kn, cos, sin, False, False)
        assert pkg.cache_struct(h).seq_len == off
    finally:
        lib.kv_cache_free(h)
    qr, kr = oracle.qk_norm_rope(q, k, qn, kn, cos, sin)
    ck = head_first(bf16_round(np.concatenate([k_old, kr])))
    cv = head_first(bf16_round(np.concatenate([v_old, v])))
    exact = oracle.chunked_prefill(bf16_round(qr), ck, cv, off)
    print(f"chunked off={off} S={S}: max {max_abs(out, exact):.3e} rel {rel_l2(out, exact):.3e}")
    assert max_abs(out, exact) <= TOL_TC_MAX and rel_l2(out, exact) <= TOL_TC_REL


def test_fused_prefill_config3(pkg, lib, oracle):
    """BASELINE config 3's shape: 4,096 tokens = 3,600 vision tokens on a 60x60 grid + 496 text
    tokens, Q/K/V ~ 0.5 N(0,1), QK-RMSNorm fused."""
    q, k, v, qn, kn, pos = _inputs(pkg, 4096, 3, grid=(60, 60, 496))
    cos, sin = oracle.mrope_cos_sin_3d(pos)
    h = new_cache(pkg, lib, 4096, pkg.ATTN_KV_BF16)
    try:
        out = _fused(pkg, lib, h, 0, q, k, v, qn, kn, cos, sin, True, True)
    finally:
        lib.kv_cache_free(h)
    exact, fp32, _ = _expect(oracle, q, k, v, qn, kn, cos, sin, True)
    print(f"config3: vs rounded max {max_abs(out, exact):.3e} rel {rel_l2(out, exact):.3e}; "
          f"vs fp32 max {max_abs(out, fp32):.3e} rel {rel_l2(out, fp32):.3e}")
    assert max_abs(out, exact) <= TOL_TC_MAX + TOL_OUT_BF16_MAX and rel_l2(out, exact) <= TOL_TC_REL + TOL_OUT_BF16_REL
    assert max_abs(out, fp32) <= TOL_TC32_MAX and rel_l2(out, fp32) <= TOL_TC32_REL


def test_fused_prefill_config5_sampled_rows(pkg, lib, oracle):
    """BASELINE config 5's prefill: 32,768 tokens = 30,000 vision tokens on a 150x200 grid + 2,768
    text tokens.  The whole page runs on the GPU; the oracle checks a sample of query rows -- the
    first and last rows, both sides of every 128-row tile edge in four regions, and random rows --
    each as causal attention over the cache rows [0, row] (the causal prefill row of
    kernel/attention.c:252-362 is that decode, :158-192, over the rows it sees), on the BF16 rows
    the kernel wrote to the cache and the BF16-rounded normalised, rotated query."""
    S = 32768
    q, k, v, qn, kn, pos = _inputs(pkg, S, 5, grid=(150, 200, 2768))
    cos, sin = oracle.mrope_cos_sin_3d(pos)
    h = new_cache(pkg, lib, S, pkg.ATTN_KV_BF16)
    try:
        out = _fused(pkg, lib, h, 13, q, k, v, qn, kn, cos, sin, False, False)
        as_f32 = lambda u: (u.astype(np.uint32) << 16).view(np.float32)  # noqa: E731
        kc = as_f32(d2h(lib.kv_cache_k(h, 13, 0), (8, S, 128), np.uint16))
        vc = as_f32(d2h(lib.kv_cache_v(h, 13, 0), (8, S, 128), np.uint16))
    finally:
        lib.kv_cache_free(h)
    qr, _ = oracle.qk_norm_rope(q, k, qn, kn, cos, sin)
    qr = bf16_round(qr)
    rng = np.random.default_rng(55)
    edges = [b + d for b in (128, 4096, 16384, 29952) for d in (-1, 0)]
    rows = sorted(set([0, 1, S - 1, 29999, 30000] + edges + list(rng.integers(0, S, 40))))
    got = np.stack([out[i] for i in rows])
    want = np.stack([oracle.decode(np.ascontiguousarray(qr[i]), kc, vc, i + 1) for i in rows])
    print(f"config5 sampled rows ({len(rows)}): max {max_abs(got, want):.3e} rel {rel_l2(got, want):.3e}")
    assert max_abs(got, want) <= TOL_TC_MAX and rel_l2(got, want) <= TOL_TC_REL


def test_fused_prefill_rejects_bad_arguments(pkg, lib):
    h = new_cache(pkg, lib, 8, pkg.ATTN_KV_F32)
    x = torch.zeros((4, 16, 128), device="cuda")
    try:
        lib.attn_clear_error()
        rc = lib.attention_prefill_fused_gqa(vp(x), vp(x), vp(x), 0, vp(x), vp(x), vp(x), vp(x), h, 0, vp(x), 0, 4,
                                             SCALE, EPS)
        assert rc != 0 and "BF16" in pkg.last_error(lib)
    finally:
        lib.attn_clear_error()
        lib.kv_cache_free(h)
    h = new_cache(pkg, lib, 8, pkg.ATTN_KV_BF16)
    try:
        host = np.zeros((4, 16, 128), dtype=np.float32)
        rc = lib.attention_prefill_fused_gqa(vp(host), vp(x), vp(x), 0, vp(x), vp(x), vp(x), vp(x), h, 0, vp(x), 0, 4,
                                             SCALE, EPS)
        assert rc != 0 and "device memory" in pkg.last_error(lib)
        lib.attn_clear_error()
        rc = lib.attention_prefill_fused_gqa(vp(x), vp(x), vp(x), 0, vp(x), vp(x), vp(x), vp(x), h, 0, vp(x), 0, 9,
                                             SCALE, EPS)
        assert rc != 0 and "exceed" in pkg.last_error(lib)
    finally:
        lib.attn_clear_error()
        lib.kv_cache_free(h)
