"""One decode step with QK-RMSNorm + M-RoPE on the GPU (attention_decode_append_fused_gqa): raw q
and k rows, the norm weights and the token's cos/sin go in; the decode kernel normalises and
rotates q and the new key row as it loads them, appends the row, and attends.  Checked against
the oracle's chain of kernel/decoder.c:73-105 (RMSNorm, M-RoPE, append, attention):
  * the key row the cache receives is the oracle's normalised, rotated row in BF16 (within one
    BF16 step: the kernel's rsqrt and the reference's estimate + Newton steps differ in the last
    FP32 bits), the value row the given one in BF16;
  * the output matches the oracle's attention over the rows the cache holds (the appended row read
    back) within the FP32 tolerance (TOL_MAX, TOL_REL) -- the BF16 path's bar when the oracle sees
    the same BF16 rows.
Lengths cover the tensor-core form (one wave) and the streaming form (long sequences)."""

import ctypes
import importlib

import numpy as np
import pytest
import torch

from gpu_helpers import TOL_MAX, TOL_REL, bf16_round, d2h, dev, fill_layer, head_first, new_cache, vp
from oracle import max_abs, rel_l2

pytestmark = pytest.mark.gpu
SCALE = ctypes.c_float(0.08838834764831843)
EPS = ctypes.c_float(1e-6)
LAYER = 2


def _step_inputs(pkg, oracle, rng, position):
    wl = importlib.import_module(pkg.__name__ + ".workloads")
    q_raw = (2.0 * rng.standard_normal((16, 128), dtype=np.float32) + 0.3).astype(np.float32)
    k_raw = (3.0 * rng.standard_normal((8, 128), dtype=np.float32)).astype(np.float32)
    v_new = rng.standard_normal((8, 128), dtype=np.float32)
    qn, kn = wl.norm_weights(rng)
    # a text token: all three M-RoPE sections at the same position (kernel/decoder.c:80-83)
    cos, sin = oracle.mrope_cos_sin_3d(np.full((3, 1), position, dtype=np.int32))
    return q_raw, k_raw, v_new, qn, kn, cos, sin


def _run(pkg, lib, h, q_raw, k_raw, v_new, qn, kn, cos, sin):
    qd, kd, vd, qnd, knd, cd, sd = (dev(x) for x in (q_raw, k_raw, v_new, qn, kn, cos, sin))
    od = torch.full((16, 128), float("nan"), dtype=torch.float32, device="cuda")
    rc = lib.attention_decode_append_fused_gqa(vp(qd), vp(kd), vp(vd), vp(qnd), vp(knd), vp(cd), vp(sd), h,
                                               vp(od), LAYER, SCALE, EPS)
    assert rc == 0, pkg.last_error(lib)
    assert lib.attn_sync() == 0, pkg.last_error(lib)
    return od.cpu().numpy()


@pytest.mark.parametrize("kv_len", [1, 17, 4097, 5000, 20001])
def test_fused_decode_step_matches_oracle_chain(pkg, lib, oracle, kv_len):
    rng = np.random.default_rng(700 + kv_len)
    max_seq = kv_len + 8
    k_old = rng.standard_normal((kv_len - 1, 8, 128), dtype=np.float32)
    v_old = rng.standard_normal((kv_len - 1, 8, 128), dtype=np.float32)
    h = new_cache(pkg, lib, max_seq, pkg.ATTN_KV_BF16)
    try:
        if kv_len > 1:
            fill_layer(pkg, lib, h, LAYER, k_old, v_old)
        pkg.cache_struct(h).seq_len = kv_len - 1
        # two steps in a row (the second at the next position), as a decode loop makes them
        outs, expect = [], []
        for step in range(2):
            n = kv_len + step
            q_raw, k_raw, v_new, qn, kn, cos, sin = _step_inputs(pkg, oracle, rng, 5000 + n)
            outs.append(_run(pkg, lib, h, q_raw, k_raw, v_new, qn, kn, cos, sin))
            qr, kr = oracle.qk_norm_rope(q_raw[None], k_raw[None], qn, kn, cos, sin)
            expect.append((qr[0], kr[0], v_new, n))
            pkg.cache_struct(h).seq_len = n  # kv_cache_advance, as decode_all_layers does
        rows_k = d2h(lib.kv_cache_k(h, LAYER, 0), (8, max_seq, 128), np.uint16)
        rows_v = d2h(lib.kv_cache_v(h, LAYER, 0), (8, max_seq, 128), np.uint16)
    finally:
        lib.kv_cache_free(h)
    as_f32 = lambda u: (u.astype(np.uint32) << 16).view(np.float32)
    k_cache, v_cache = as_f32(rows_k), as_f32(rows_v)  # head-first [8, max_seq, 128]
    for out, (qr, kr, v_new, n) in zip(outs, expect):
        got_k = k_cache[:, n - 1]
        want_k = bf16_round(kr)
        # within one BF16 step of the oracle's row (relative 2^-7 covers a last-bit tie)
        assert np.all(np.abs(got_k - want_k) <= np.abs(want_k) * 2.0 ** -7 + 1e-30), "appended K row"
        assert np.array_equal(v_cache[:, n - 1], bf16_round(v_new)), "appended V row"
        exact = oracle.decode(qr, k_cache, v_cache, n)
        print(f"kv_len {n}: max {max_abs(out, exact):.3e} rel {rel_l2(out, exact):.3e}")
        assert max_abs(out, exact) <= TOL_MAX and rel_l2(out, exact) <= TOL_REL


def test_fused_decode_rejects_what_it_cannot_take(pkg, lib, oracle):
    rng = np.random.default_rng(9)
    q_raw, k_raw, v_new, qn, kn, cos, sin = _step_inputs(pkg, oracle, rng, 12)
    f32 = new_cache(pkg, lib, 64, pkg.ATTN_KV_F32)
    b16 = new_cache(pkg, lib, 64, pkg.ATTN_KV_BF16)
    try:
        pkg.cache_struct(f32).seq_len = 10
        pkg.cache_struct(b16).seq_len = 10
        qd, kd, vd, qnd, knd, cd, sd = (dev(x) for x in (q_raw, k_raw, v_new, qn, kn, cos, sin))
        od = torch.zeros((16, 128), dtype=torch.float32, device="cuda")
        lib.attn_clear_error()
        rc = lib.attention_decode_append_fused_gqa(vp(qd), vp(kd), vp(vd), vp(qnd), vp(knd), vp(cd), vp(sd), f32,
                                                   vp(od), LAYER, SCALE, EPS)
        assert rc != 0 and "BF16" in pkg.last_error(lib)
        lib.attn_clear_error()
        host_q = np.ascontiguousarray(q_raw)
        rc = lib.attention_decode_append_fused_gqa(host_q.ctypes.data, vp(kd), vp(vd), vp(qnd), vp(knd), vp(cd),
                                                   vp(sd), b16, vp(od), LAYER, SCALE, EPS)
        assert rc != 0 and "device memory" in pkg.last_error(lib)
        lib.attn_clear_error()
        pkg.cache_struct(b16).seq_len = 64  # no row left to append into
        rc = lib.attention_decode_append_fused_gqa(vp(qd), vp(kd), vp(vd), vp(qnd), vp(knd), vp(cd), vp(sd), b16,
                                                   vp(od), LAYER, SCALE, EPS)
        assert rc != 0 and "max_seq_len" in pkg.last_error(lib)
        lib.attn_clear_error()
    finally:
        lib.kv_cache_free(f32)
        lib.kv_cache_free(b16)
