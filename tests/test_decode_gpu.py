"""Split-KV decode kernel vs the oracle (kernel/attention.c:158-204 semantics), through
the C-ABI entry points attention_decode_gqa and attention_decode_gqa_batched."""

import ctypes

import numpy as np
import pytest
import torch

from gpu_helpers import (TOL_BF16_MAX, TOL_BF16_REL, TOL_MAX, TOL_REL, bf16_round, check, dev, fill_layer,
                         head_first, new_cache, vp)
from oracle import max_abs, rel_l2

pytestmark = pytest.mark.gpu
SCALE = ctypes.c_float(0.08838834764831843)


def _run_decode(pkg, lib, h, q, layer, kv_len, on_device):
    if on_device:
        qd = dev(q)
        od = torch.zeros((16, 128), dtype=torch.float32, device="cuda")
        lib.attention_decode_gqa(vp(qd), h, vp(od), layer, kv_len, SCALE)
        assert lib.attn_sync() == 0, pkg.last_error(lib)
        check(pkg, lib, "decode")
        return od.cpu().numpy()
    out = np.zeros((16, 128), dtype=np.float32)
    lib.attention_decode_gqa(vp(q), h, vp(out), layer, kv_len, SCALE)
    check(pkg, lib, "decode")
    return out


def test_golden_decode(pkg, lib, golden):
    g = golden("decode_kv45.npz")
    n = g["k_rows"].shape[0]
    h = new_cache(pkg, lib, 64, pkg.ATTN_KV_F32)
    try:
        fill_layer(pkg, lib, h, 3, g["k_rows"], g["v_rows"])
        out = _run_decode(pkg, lib, h, g["q"], 3, n, on_device=False)
        assert max_abs(out, g["out"]) <= TOL_MAX and rel_l2(out, g["out"]) <= TOL_REL
    finally:
        lib.kv_cache_free(h)


@pytest.mark.parametrize("kv_len", [1, 2, 15, 16, 17, 63, 64, 65, 127, 128, 129, 1000, 4097, 8192])
@pytest.mark.parametrize("on_device", [False, True])
def test_decode_fp32_vs_oracle(pkg, lib, oracle, kv_len, on_device):
    rng = np.random.default_rng(kv_len)
    max_seq = kv_len + 5
    q = rng.standard_normal((16, 128), dtype=np.float32)
    k = rng.standard_normal((max_seq, 8, 128), dtype=np.float32)
    v = rng.standard_normal((max_seq, 8, 128), dtype=np.float32)
    h = new_cache(pkg, lib, max_seq, pkg.ATTN_KV_F32)
    try:
        fill_layer(pkg, lib, h, 27, k, v)
        out = _run_decode(pkg, lib, h, q, 27, kv_len, on_device)
    finally:
        lib.kv_cache_free(h)
    want = oracle.decode(q, head_first(k), head_first(v), kv_len)
    assert max_abs(out, want) <= TOL_MAX and rel_l2(out, want) <= TOL_REL


@pytest.mark.parametrize("kv_len", [1, 33, 129, 4097])
def test_decode_bf16_cache(pkg, lib, oracle, kv_len):
    rng = np.random.default_rng(100 + kv_len)
    q = rng.standard_normal((16, 128), dtype=np.float32)
    k = rng.standard_normal((kv_len, 8, 128), dtype=np.float32)
    v = rng.standard_normal((kv_len, 8, 128), dtype=np.float32)
    h = new_cache(pkg, lib, kv_len, pkg.ATTN_KV_BF16)
    try:
        fill_layer(pkg, lib, h, 0, k, v)
        out = _run_decode(pkg, lib, h, q, 0, kv_len, on_device=True)
    finally:
        lib.kv_cache_free(h)
    # Same rows the kernel holds (bf16-rounded): the FP32 bar applies.
    exact = oracle.decode(q, head_first(bf16_round(k)), head_first(bf16_round(v)), kv_len)
    assert max_abs(out, exact) <= TOL_MAX and rel_l2(out, exact) <= TOL_REL
    # Against the FP32 reference inputs: the stated BF16 KV tolerance.
    ref32 = oracle.decode(q, head_first(k), head_first(v), kv_len)
    assert max_abs(out, ref32) <= TOL_BF16_MAX and rel_l2(out, ref32) <= TOL_BF16_REL


def test_decode_repeated_calls_reuse_workspace(pkg, lib, oracle):
    """Split tickets must be left at zero: alternate long/short calls on one cache."""
    rng = np.random.default_rng(7)
    n = 3000
    k = rng.standard_normal((n, 8, 128), dtype=np.float32)
    v = rng.standard_normal((n, 8, 128), dtype=np.float32)
    h = new_cache(pkg, lib, n, pkg.ATTN_KV_F32)
    try:
        fill_layer(pkg, lib, h, 1, k, v)
        for kv_len in (3000, 40, 2999, 1, 1777, 3000):
            q = rng.standard_normal((16, 128), dtype=np.float32)
            out = _run_decode(pkg, lib, h, q, 1, kv_len, on_device=bool(kv_len % 2))
            want = oracle.decode(q, head_first(k), head_first(v), kv_len)
            assert max_abs(out, want) <= TOL_MAX, kv_len
    finally:
        lib.kv_cache_free(h)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_decode_batched_ragged(pkg, lib, oracle, dtype):
    rng = np.random.default_rng(11)
    lens = [1, 17, 300, 1024, 2049, 5000]
    kv_dt = pkg.ATTN_KV_F32 if dtype == "f32" else pkg.ATTN_KV_BF16
    caches, rows = [], []
    try:
        for L in lens:
            h = new_cache(pkg, lib, L + 8, kv_dt)
            caches.append(h)
            k = rng.standard_normal((L, 8, 128), dtype=np.float32)
            v = rng.standard_normal((L, 8, 128), dtype=np.float32)
            fill_layer(pkg, lib, h, 5, k, v)
            rows.append((k, v))
        q = rng.standard_normal((len(lens), 16, 128), dtype=np.float32)
        out = np.zeros_like(q)
        arr = (ctypes.c_void_p * len(lens))(*caches)
        kvl = (ctypes.c_int * len(lens))(*lens)
        rc = lib.attention_decode_gqa_batched(vp(q), arr, kvl, vp(out), len(lens), 5, SCALE)
        assert rc == 0, pkg.last_error(lib)
    finally:
        for h in caches:
            lib.kv_cache_free(h)
    for b, (L, (k, v)) in enumerate(zip(lens, rows)):
        if dtype == "bf16":
            k, v = bf16_round(k), bf16_round(v)
        want = oracle.decode(q[b], head_first(k), head_first(v), L)
        assert max_abs(out[b], want) <= TOL_MAX and rel_l2(out[b], want) <= TOL_REL, (b, L)


def test_decode_kv_len_zero_gives_zeros(pkg, lib):
    h = new_cache(pkg, lib, 16, pkg.ATTN_KV_F32)
    try:
        out = np.full((16, 128), 7.0, dtype=np.float32)
        q = np.ones((16, 128), dtype=np.float32)
        lib.attention_decode_gqa(vp(q), h, vp(out), 0, 0, SCALE)
        check(pkg, lib, "decode kv_len 0")
        assert not out.any()
    finally:
        lib.kv_cache_free(h)


def test_decode_rejects_bad_arguments(pkg, lib):
    h = new_cache(pkg, lib, 16, pkg.ATTN_KV_F32)
    try:
        q = np.ones((16, 128), dtype=np.float32)
        out = np.zeros((16, 128), dtype=np.float32)
        for layer, kv_len in ((28, 4), (-1, 4), (0, 17), (0, -2)):
            lib.attn_clear_error()
            lib.attention_decode_gqa(vp(q), h, vp(out), layer, kv_len, SCALE)
            assert pkg.last_error(lib), (layer, kv_len)
        lib.attn_clear_error()
        bogus = ctypes.create_string_buffer(8192)
        lib.attention_decode_gqa(vp(q), ctypes.addressof(bogus), vp(out), 0, 1, SCALE)
        assert "not allocated" in pkg.last_error(lib)
        lib.attn_clear_error()
    finally:
        lib.kv_cache_free(h)


def _oracle_rows(k_rows, v_rows, n):
    return head_first(k_rows[:n]), head_first(v_rows[:n])


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("pos", [0, 1, 63, 64, 700, 4096])
def test_decode_append_fused(pkg, lib, oracle, dtype, pos):
    """attention_decode_append_gqa == kv_cache_append + attention_decode_gqa(kv_len = pos + 1)."""
    kv_dt = pkg.ATTN_KV_F32 if dtype == "f32" else pkg.ATTN_KV_BF16
    rng = np.random.default_rng(900 + pos)
    rows = pos + 1
    k = rng.standard_normal((rows, 8, 128), dtype=np.float32)
    v = rng.standard_normal((rows, 8, 128), dtype=np.float32)
    q = rng.standard_normal((16, 128), dtype=np.float32)
    h = new_cache(pkg, lib, rows + 2, kv_dt)
    try:
        if pos:
            fill_layer(pkg, lib, h, 2, k[:pos], v[:pos])
        pkg.cache_struct(h).seq_len = pos
        out = np.zeros((16, 128), dtype=np.float32)
        rc = lib.attention_decode_append_gqa(vp(q), vp(k[pos]), vp(v[pos]), h, vp(out), 2, SCALE)
        assert rc == 0, pkg.last_error(lib)
        assert pkg.cache_struct(h).seq_len == pos  # not advanced, as in the reference
        from gpu_helpers import d2h
        esz = np.float32 if dtype == "f32" else np.uint16
        got_k = d2h(lib.kv_cache_k(h, 2, 5) + pos * 128 * (4 if dtype == "f32" else 2), (128,), esz)
        if dtype == "bf16":
            got_k = (got_k.astype(np.uint32) << 16).view(np.float32)
            assert np.array_equal(got_k, bf16_round(k[pos, 5]))
        else:
            assert np.array_equal(got_k, k[pos, 5])
    finally:
        lib.kv_cache_free(h)
    kk, vv = (bf16_round(k), bf16_round(v)) if dtype == "bf16" else (k, v)
    want = oracle.decode(q, head_first(kk), head_first(vv), rows)
    assert max_abs(out, want) <= TOL_MAX and rel_l2(out, want) <= TOL_REL


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_decode_steps_device_queue(pkg, lib, oracle, dtype):
    """Several decode steps over 4 layers, device pointers, no host sync between calls:
    each launch may stream older rows before its predecessor finishes, so this checks
    that rows the previous launch wrote are never read early."""
    kv_dt = pkg.ATTN_KV_F32 if dtype == "f32" else pkg.ATTN_KV_BF16
    rng = np.random.default_rng(77)
    layers, pre, steps = 4, 300, 5
    max_seq = pre + steps
    ks = rng.standard_normal((layers, max_seq, 8, 128), dtype=np.float32)
    vs = rng.standard_normal((layers, max_seq, 8, 128), dtype=np.float32)
    qs = rng.standard_normal((steps, layers, 16, 128), dtype=np.float32)
    h = new_cache(pkg, lib, max_seq, kv_dt)
    outs = torch.zeros((steps, layers, 16, 128), dtype=torch.float32, device="cuda")
    kd, vd, qd = dev(ks), dev(vs), dev(qs)
    try:
        for layer in range(layers):
            fill_layer(pkg, lib, h, layer, ks[layer, :pre], vs[layer, :pre])
        cs = pkg.cache_struct(h)
        cs.seq_len = pre
        for s in range(steps):
            for layer in range(layers):
                pos = pre + s
                rc = lib.attention_decode_append_gqa(
                    ctypes.c_void_p(qd[s, layer].data_ptr()), ctypes.c_void_p(kd[layer, pos].data_ptr()),
                    ctypes.c_void_p(vd[layer, pos].data_ptr()), h, ctypes.c_void_p(outs[s, layer].data_ptr()),
                    layer, SCALE)
                assert rc == 0, pkg.last_error(lib)
                # Same layer again right away (plain decode over the row just written).
                if layer == 1:
                    lib.attention_decode_gqa(ctypes.c_void_p(qd[s, 0].data_ptr()), h,
                                             ctypes.c_void_p(outs[s, 0].data_ptr()), 1, pos + 1, SCALE)
            lib.kv_cache_advance(h, 1)
        assert lib.attn_sync() == 0, pkg.last_error(lib)
        got = outs.cpu().numpy()
    finally:
        lib.kv_cache_free(h)
    if dtype == "bf16":
        ks, vs = bf16_round(ks), bf16_round(vs)
    for s in range(steps):
        rows = pre + s + 1
        for layer in range(layers):
            qq = qs[s, 0] if layer == 0 else qs[s, layer]
            src = 1 if layer == 0 else layer  # slot 0 was overwritten by the repeat on layer 1
            want = oracle.decode(qq, head_first(ks[src, :rows]), head_first(vs[src, :rows]), rows)
            assert max_abs(got[s, layer], want) <= TOL_MAX and rel_l2(got[s, layer], want) <= TOL_REL, (s, layer)


def test_decode_long_context_bf16(pkg, lib, oracle):
    """Config 5's decode length (32,768 prefilled + 1,024): 16-CTA clusters, many stages."""
    kv_len = 33792
    rng = np.random.default_rng(5)
    k = (0.5 * rng.standard_normal((kv_len, 8, 128), dtype=np.float32)).astype(np.float32)
    v = (0.5 * rng.standard_normal((kv_len, 8, 128), dtype=np.float32)).astype(np.float32)
    q = rng.standard_normal((16, 128), dtype=np.float32)
    h = new_cache(pkg, lib, kv_len, pkg.ATTN_KV_BF16)
    try:
        fill_layer(pkg, lib, h, 27, k, v)
        out = _run_decode(pkg, lib, h, q, 27, kv_len, on_device=True)
    finally:
        lib.kv_cache_free(h)
    want = oracle.decode(q, head_first(bf16_round(k)), head_first(bf16_round(v)), kv_len)
    assert max_abs(out, want) <= TOL_MAX and rel_l2(out, want) <= TOL_REL


def _pinned(a):
    """A page-locked host copy of `a` (the decode entry points read and write such buffers in
    place through their device mapping instead of copying them)."""
    t = torch.from_numpy(np.ascontiguousarray(a)).pin_memory()
    assert t.is_pinned()
    return t


@pytest.mark.parametrize("kv_len", [0, 1, 129, 4097])
def test_decode_pinned_host_buffers(pkg, lib, oracle, kv_len):
    rng = np.random.default_rng(5000 + kv_len)
    max_seq = kv_len + 3
    q = rng.standard_normal((16, 128), dtype=np.float32)
    k = rng.standard_normal((max_seq, 8, 128), dtype=np.float32)
    v = rng.standard_normal((max_seq, 8, 128), dtype=np.float32)
    h = new_cache(pkg, lib, max_seq, pkg.ATTN_KV_F32)
    try:
        fill_layer(pkg, lib, h, 11, k, v)
        qp, op = _pinned(q), _pinned(np.full((16, 128), 3.0, dtype=np.float32))
        lib.attention_decode_gqa(vp(qp), h, vp(op), 11, kv_len, SCALE)
        check(pkg, lib, "decode pinned")
        out_pinned = op.numpy().copy()
        # page-locked input with a pageable output, and the reverse
        out_mixed = np.zeros((16, 128), dtype=np.float32)
        lib.attention_decode_gqa(vp(qp), h, vp(out_mixed), 11, kv_len, SCALE)
        check(pkg, lib, "decode pinned q")
        op2 = _pinned(np.zeros((16, 128), dtype=np.float32))
        lib.attention_decode_gqa(vp(q), h, vp(op2), 11, kv_len, SCALE)
        check(pkg, lib, "decode pinned out")
    finally:
        lib.kv_cache_free(h)
    if kv_len == 0:
        want = np.zeros((16, 128), dtype=np.float32)
        assert not out_pinned.any() and not out_mixed.any() and not op2.numpy().any()
        return
    want = oracle.decode(q, head_first(k), head_first(v), kv_len)
    for got in (out_pinned, out_mixed, op2.numpy()):
        assert max_abs(got, want) <= TOL_MAX and rel_l2(got, want) <= TOL_REL


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("pos", [0, 700, 4096])
def test_decode_append_pinned_host_buffers(pkg, lib, oracle, dtype, pos):
    kv_dt = pkg.ATTN_KV_F32 if dtype == "f32" else pkg.ATTN_KV_BF16
    rng = np.random.default_rng(7000 + pos)
    rows = pos + 1
    k = rng.standard_normal((rows, 8, 128), dtype=np.float32)
    v = rng.standard_normal((rows, 8, 128), dtype=np.float32)
    q = rng.standard_normal((16, 128), dtype=np.float32)
    h = new_cache(pkg, lib, rows + 2, kv_dt)
    try:
        if pos:
            fill_layer(pkg, lib, h, 7, k[:pos], v[:pos])
        pkg.cache_struct(h).seq_len = pos
        qp, kp, vp_, op = _pinned(q), _pinned(k[pos]), _pinned(v[pos]), _pinned(np.zeros((16, 128), np.float32))
        rc = lib.attention_decode_append_gqa(vp(qp), vp(kp), vp(vp_), h, vp(op), 7, SCALE)
        assert rc == 0, pkg.last_error(lib)
        out = op.numpy().copy()
        # the appended row reads back from the cache as written
        rc = lib.attention_decode_append_gqa(vp(q), vp(k[pos]), vp(v[pos]), h, vp(op), 7, SCALE)
        assert rc == 0, pkg.last_error(lib)
        again = op.numpy().copy()
    finally:
        lib.kv_cache_free(h)
    kk, vv = (bf16_round(k), bf16_round(v)) if dtype == "bf16" else (k, v)
    want = oracle.decode(q, head_first(kk), head_first(vv), rows)
    assert max_abs(out, want) <= TOL_MAX and rel_l2(out, want) <= TOL_REL
    assert np.array_equal(out, again)


def _plan(lib, kv_len, dtype):
    chunk, nsplit = ctypes.c_int(), ctypes.c_int()
    lib.tyb_decode_plan(1, kv_len, dtype, ctypes.byref(chunk), ctypes.byref(nsplit))
    return chunk.value, nsplit.value


def _edge_lengths(pkg, lib):
    """kv lengths around 16-row steps and split edges of the BF16 single-sequence kernels
    (one wave of splits up to 4,608 rows, streamed spans past it), including ones whose last
    split holds only the appended row."""
    lens = {1, 2, 15, 16, 17, 100, 191, 192, 193, 2000, 4097, 4608, 8192,
            4609, 12289, 20001}  # past one wave: the streaming form (64-row stages, spans)
    for target in (300, 2000, 4097):
        chunk, _ = _plan(lib, target, pkg.ATTN_KV_BF16)
        n = (target // chunk) * chunk + 1
        if _plan(lib, n, pkg.ATTN_KV_BF16)[0] == chunk:
            lens.add(n)
    return sorted(lens)


@pytest.mark.parametrize("append", [False, True])
def test_decode_bf16_split_edges(pkg, lib, oracle, append):
    """BF16 cache, one sequence (the tensor-core form): every split/step edge against the
    oracle on the same bf16-rounded rows, FP32 bar; NaN in the slab past the attended rows."""
    lib.tyb_decode_plan.restype = None
    for kv_len in _edge_lengths(pkg, lib):
        rng = np.random.default_rng(5000 + kv_len)
        q = rng.standard_normal((16, 128), dtype=np.float32)
        k = rng.standard_normal((kv_len, 8, 128), dtype=np.float32)
        v = rng.standard_normal((kv_len, 8, 128), dtype=np.float32)
        h = new_cache(pkg, lib, kv_len + 40, pkg.ATTN_KV_BF16)
        try:
            qd = dev(q)
            od = torch.full((16, 128), float("nan"), dtype=torch.float32, device="cuda")
            # Rows past the attended ones (the appended row's slot included) hold NaN: the
            # kernel reads whole tiles and must not let them in.
            n_old = kv_len - 1 if append else kv_len
            pad = np.full((kv_len + 40, 8, 128), np.nan, dtype=np.float32)
            kf, vf = pad.copy(), pad.copy()
            kf[:n_old], vf[:n_old] = k[:n_old], v[:n_old]
            fill_layer(pkg, lib, h, 4, kf, vf)
            if append:
                pkg.cache_struct(h).seq_len = kv_len - 1
                kn, vn = dev(k[kv_len - 1]), dev(v[kv_len - 1])
                rc = lib.attention_decode_append_gqa(vp(qd), vp(kn), vp(vn), h, vp(od), 4, SCALE)
                assert rc == 0, pkg.last_error(lib)
            else:
                lib.attention_decode_gqa(vp(qd), h, vp(od), 4, kv_len, SCALE)
            assert lib.attn_sync() == 0, pkg.last_error(lib)
            check(pkg, lib, "decode")
            out = od.cpu().numpy()
        finally:
            lib.kv_cache_free(h)
        want = oracle.decode(q, head_first(bf16_round(k)), head_first(bf16_round(v)), kv_len)
        assert np.isfinite(out).all(), kv_len
        assert max_abs(out, want) <= TOL_MAX and rel_l2(out, want) <= TOL_REL, kv_len


def test_decode_batched_bf16_edges_nan_tail(pkg, lib, oracle):
    """Request batch over BF16 caches (the tensor-core form with per-sequence tensor maps):
    lengths at 16-row and split edges, NaN rows past every sequence's length, device buffers,
    two calls in a row (tickets reset), one cache used by two sequences."""
    rng = np.random.default_rng(23)
    lens = [1, 15, 16, 17, 191, 192, 193, 385, 1000, 4097, 8191]
    caches, rows = [], []
    try:
        for L in lens:
            h = new_cache(pkg, lib, L + 40, pkg.ATTN_KV_BF16)
            caches.append(h)
            k = np.full((L + 40, 8, 128), np.nan, dtype=np.float32)
            v = np.full((L + 40, 8, 128), np.nan, dtype=np.float32)
            k[:L] = rng.standard_normal((L, 8, 128), dtype=np.float32)
            v[:L] = rng.standard_normal((L, 8, 128), dtype=np.float32)
            fill_layer(pkg, lib, h, 9, k, v)
            rows.append((k[:L], v[:L]))
        # the last sequence reads the first cache again, shorter
        lens_all = lens + [1]
        cache_all = caches + [caches[0]]
        rows_all = rows + [rows[0]]
        n = len(lens_all)
        arr = (ctypes.c_void_p * n)(*cache_all)
        kvl = (ctypes.c_int * n)(*lens_all)
        for call in range(2):
            q = rng.standard_normal((n, 16, 128), dtype=np.float32)
            qd = dev(q)
            od = torch.full((n, 16, 128), float("nan"), dtype=torch.float32, device="cuda")
            rc = lib.attention_decode_gqa_batched(vp(qd), arr, kvl, vp(od), n, 9, SCALE)
            assert rc == 0, pkg.last_error(lib)
            assert lib.attn_sync() == 0, pkg.last_error(lib)
            out = od.cpu().numpy()
            for b, (L, (k, v)) in enumerate(zip(lens_all, rows_all)):
                want = oracle.decode(q[b], head_first(bf16_round(k)), head_first(bf16_round(v)), L)
                assert np.isfinite(out[b]).all(), (call, b, L)
                assert max_abs(out[b], want) <= TOL_MAX and rel_l2(out[b], want) <= TOL_REL, (call, b, L)
    finally:
        for h in caches:
            lib.kv_cache_free(h)
