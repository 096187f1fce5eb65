"""Config 1 as one chain: a 1,024-token prefill (768 vision tokens on a 24x32 M-RoPE grid + 256
text tokens) followed by 256 decode steps that append to the static cache while rope_offset
advances -- the sequence kernel/decoder.c runs for one layer (:73-117 prefill, :73-105 per decode
step), with the cache bookkeeping of kernel/kv_cache.c:106-110 (kv_cache_advance) and the
rope_offset that decoder.py:428-430 sets after the prefill (max position + 1).

Two forms, each step compared with the oracle running the same chain:
  * the drop-in form: host QK-RMSNorm + M-RoPE (the oracle standing in for kernel/ops.c, as the
    unmodified decoder.c runs them on the host), then this library's kv_cache_append_prefill,
    attention_prefill_gqa, kv_cache_append, attention_decode_gqa and kv_cache_advance on an FP32
    cache with host buffers -- the FP32 bar (TOL_MAX, TOL_REL) at every step;
  * the device form: attention_prefill_fused_gqa and attention_decode_append_fused_gqa on a BF16
    cache (norm, rotation, append and attention on the GPU) -- every decode step within the FP32
    bar of the oracle run over the rows the cache holds, the prefill within the BF16 tensor-core
    bar.
"""

import ctypes
import importlib

import numpy as np
import pytest
import torch

from gpu_helpers import TOL_MAX, TOL_REL, bf16_round, check, d2h, dev, new_cache, vp
from oracle import max_abs, rel_l2

pytestmark = pytest.mark.gpu
SCALE = ctypes.c_float(0.08838834764831843)
EPS = ctypes.c_float(1e-6)
LAYER = 7
# the tensor-core prefill against the oracle fed the same BF16-rounded operands (the bar of
# test_prefill_tc_gpu.py; measured here 1.5e-3 / 1.2e-3)
TOL_TC_MAX, TOL_TC_REL = 4e-3, 2.6e-3


def _config1(pkg):
    wl = importlib.import_module(pkg.__name__ + ".workloads")
    return wl.config1(seed=0, n_decode=256)


def _decode_position(cs):
    """kernel/decoder.c:80-83: rope_offset when set, else seq_len."""
    return cs.rope_offset if cs.rope_offset else cs.seq_len


def test_config1_chain_dropin_fp32(pkg, lib, oracle):
    c = _config1(pkg)
    S, n_dec = c["q"].shape[0], len(c["decode"])
    max_seq = S + n_dec
    cos, sin = oracle.mrope_cos_sin_3d(c["pos"])
    q, k = oracle.qk_norm_rope(c["q"], c["k"], c["q_norm"], c["k_norm"], cos, sin)
    v = c["v"]
    tab_c, tab_s = oracle.mrope_table(c["rope_offset"] + n_dec + 1)
    h = lib.kv_cache_alloc(max_seq)  # the reference's FP32 cache (decoder_cache_alloc)
    assert h, pkg.last_error(lib)
    cs = pkg.cache_struct(h)
    kc = np.zeros((8, max_seq, 128), dtype=np.float32)  # the oracle's copy of the layer, head-first
    vc = np.zeros_like(kc)
    worst = [0.0, 0.0]
    try:
        lib.kv_cache_append_prefill(h, LAYER, vp(k), vp(v), S)
        out = np.zeros_like(q)
        lib.attention_prefill_gqa(vp(q), vp(k), vp(v), vp(out), S, S, SCALE, None, None, None, None)
        check(pkg, lib, "prefill")
        want = oracle.prefill(q, k, v)
        assert max_abs(out, want) <= TOL_MAX and rel_l2(out, want) <= TOL_REL
        kc[:, :S], vc[:, :S] = k.transpose(1, 0, 2), v.transpose(1, 0, 2)
        lib.kv_cache_advance(h, S)
        assert cs.seq_len == S and cs.rope_offset == 0  # rope_offset moves only once set
        cs.rope_offset = c["rope_offset"]  # decoder_cache_set_rope_offset (decoder.c:347-350)
        for i, (qs, ks, vs) in enumerate(c["decode"]):
            p = _decode_position(cs)
            qd, kd = oracle.qk_norm_rope(qs, ks, c["q_norm"], c["k_norm"], tab_c[p:p + 1], tab_s[p:p + 1])
            qd, kd, vd = qd[0], kd[0], np.ascontiguousarray(vs[0])
            n = cs.seq_len
            lib.kv_cache_append(h, LAYER, vp(kd), vp(vd))
            od = np.zeros((16, 128), dtype=np.float32)
            lib.attention_decode_gqa(vp(qd), h, vp(od), LAYER, n + 1, SCALE)
            check(pkg, lib, f"decode step {i}")
            kc[:, n], vc[:, n] = kd, vd
            want = oracle.decode(qd, kc, vc, n + 1)
            e_max, e_rel = max_abs(od, want), rel_l2(od, want)
            worst = [max(worst[0], e_max), max(worst[1], e_rel)]
            assert e_max <= TOL_MAX and e_rel <= TOL_REL, (i, e_max, e_rel)
            lib.kv_cache_advance(h, 1)
        assert cs.seq_len == S + n_dec and cs.rope_offset == c["rope_offset"] + n_dec
        # the cache holds exactly the rows the chain appended
        got_k = d2h(lib.kv_cache_k(h, LAYER, 3), (max_seq, 128))
        assert np.array_equal(got_k, kc[3])
    finally:
        lib.kv_cache_free(h)
    print(f"config1 drop-in chain: worst decode step max {worst[0]:.3e} rel {worst[1]:.3e}")


def test_config1_chain_fused_bf16(pkg, lib, oracle):
    c = _config1(pkg)
    S, n_dec = c["q"].shape[0], len(c["decode"])
    max_seq = S + n_dec
    cos, sin = oracle.mrope_cos_sin_3d(c["pos"])
    tab_c, tab_s = oracle.mrope_table(c["rope_offset"] + n_dec + 1)
    h = new_cache(pkg, lib, max_seq, pkg.ATTN_KV_BF16)
    cs = pkg.cache_struct(h)
    outs = []
    try:
        t = [dev(x) for x in (c["q"], c["k"], c["v"], c["q_norm"], c["k_norm"], cos, sin)]
        op = torch.zeros((S, 16, 128), device="cuda")
        rc = lib.attention_prefill_fused_gqa(vp(t[0]), vp(t[1]), vp(t[2]), pkg.ATTN_DT_F32, vp(t[3]), vp(t[4]),
                                             vp(t[5]), vp(t[6]), h, LAYER, vp(op), pkg.ATTN_DT_F32, S, SCALE, EPS)
        assert rc == 0, pkg.last_error(lib)
        lib.kv_cache_advance(h, S)
        cs.rope_offset = c["rope_offset"]
        qn_d, kn_d = t[3], t[4]
        steps = []
        for i, (qs, ks, vs) in enumerate(c["decode"]):
            p = _decode_position(cs)
            cd, sd = dev(tab_c[p]), dev(tab_s[p])
            qd, kd, vd = dev(qs[0]), dev(ks[0]), dev(vs[0])
            od = torch.full((16, 128), float("nan"), device="cuda")
            rc = lib.attention_decode_append_fused_gqa(vp(qd), vp(kd), vp(vd), vp(qn_d), vp(kn_d), vp(cd), vp(sd), h,
                                                       vp(od), LAYER, SCALE, EPS)
            assert rc == 0, (i, pkg.last_error(lib))
            outs.append(od)
            steps.append((p, cs.seq_len))
            lib.kv_cache_advance(h, 1)
        assert lib.attn_sync() == 0, pkg.last_error(lib)
        pre = op.cpu().numpy()
        outs = [o.cpu().numpy() for o in outs]
        as_f32 = lambda u: (u.astype(np.uint32) << 16).view(np.float32)  # noqa: E731
        kc = as_f32(d2h(lib.kv_cache_k(h, LAYER, 0), (8, max_seq, 128), np.uint16))
        vc = as_f32(d2h(lib.kv_cache_v(h, LAYER, 0), (8, max_seq, 128), np.uint16))
    finally:
        lib.kv_cache_free(h)
    assert cs.seq_len == S + n_dec and cs.rope_offset == c["rope_offset"] + n_dec
    # prefill: against the oracle chain on the same BF16-rounded normalised, rotated operands
    qr, kr = oracle.qk_norm_rope(c["q"], c["k"], c["q_norm"], c["k_norm"], cos, sin)
    want = oracle.prefill(bf16_round(qr), bf16_round(kr), bf16_round(c["v"]))
    print(f"config1 fused prefill: max {max_abs(pre, want):.3e} rel {rel_l2(pre, want):.3e}")
    assert max_abs(pre, want) <= TOL_TC_MAX and rel_l2(pre, want) <= TOL_TC_REL
    # every cache row the prefill wrote is the oracle's row in BF16: within one BF16 step, plus
    # an absolute 1e-5 for rotated values that cancel to near zero (the kernel's rsqrt and the
    # reference's estimate + Newton steps differ in the last FP32 bits)
    want_k = bf16_round(kr).transpose(1, 0, 2)
    assert np.all(np.abs(kc[:, :S] - want_k) <= np.abs(want_k) * 2.0 ** -7 + 1e-5)
    assert np.array_equal(vc[:, :S], bf16_round(c["v"]).transpose(1, 0, 2))
    worst = [0.0, 0.0]
    for i, ((qs, ks, vs), (p, n), out) in enumerate(zip(c["decode"], steps, outs)):
        qd, kd = oracle.qk_norm_rope(qs, ks, c["q_norm"], c["k_norm"], tab_c[p:p + 1], tab_s[p:p + 1])
        assert np.all(np.abs(kc[:, n] - bf16_round(kd[0])) <= np.abs(bf16_round(kd[0])) * 2.0 ** -7 + 1e-5), i
        want = oracle.decode(qd[0], kc, vc, n + 1)
        e_max, e_rel = max_abs(out, want), rel_l2(out, want)
        worst = [max(worst[0], e_max), max(worst[1], e_rel)]
        assert e_max <= TOL_MAX and e_rel <= TOL_REL, (i, e_max, e_rel)
    print(f"config1 fused chain: worst decode step max {worst[0]:.3e} rel {worst[1]:.3e}")
