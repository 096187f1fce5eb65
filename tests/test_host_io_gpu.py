"""Decode calls with host inputs and outputs, as kernel/decoder.c:96-105 makes them every step (q,
the new K/V row and the attention output in host buffers, the call returning with the output
written).  Host inputs travel as the launch's own parameter block (copied into the layer's
page-locked slot, which the launch reads as its parameters), and a host output is stored by the
kernel through a device mapping -- the caller's page-locked buffer in place, a pageable one by way
of the cache's page-locked staging -- after the host has filled it with a NaN pattern that GPU
arithmetic never produces; the call returns once no word holds it.

Checked here: every combination of input and output residency (device, page-locked, pageable)
gives the same bits as device buffers, on each kernel form a call can reach (FP32 split kernel,
BF16 tensor-core splits up to 4,608 rows, BF16 streaming spans beyond), for the full call, the
KV-head subsets, the plain decode without an append and the deferred append of decoder.c; and
calls back to back keep returning their own results."""

import ctypes

import numpy as np
import pytest
import torch

from gpu_helpers import fill_layer, new_cache, vp

pytestmark = pytest.mark.gpu
SCALE = ctypes.c_float(0.08838834764831843)
LAYER = 3


def _buf(kind, shape, src=None):
    """(buffer, pointer) of `kind`: device tensor, page-locked host tensor or numpy array."""
    if kind == "device":
        t = torch.zeros(shape, dtype=torch.float32, device="cuda")
        if src is not None:
            t.copy_(torch.from_numpy(src))
        return t, ctypes.c_void_p(t.data_ptr())
    if kind == "pinned":
        t = torch.zeros(shape, dtype=torch.float32).pin_memory()
        if src is not None:
            t.copy_(torch.from_numpy(src))
        return t, ctypes.c_void_p(t.data_ptr())
    a = np.zeros(shape, dtype=np.float32) if src is None else np.ascontiguousarray(src.copy())
    return a, vp(a)


def _read(buf):
    if isinstance(buf, np.ndarray):
        return buf.copy()
    return buf.cpu().numpy().copy()


def _setup(pkg, lib, dtype, n, seed):
    rng = np.random.default_rng(seed)
    h = new_cache(pkg, lib, n + 8, dtype)
    k = rng.standard_normal((n, 8, 128), dtype=np.float32)
    v = rng.standard_normal((n, 8, 128), dtype=np.float32)
    if n:
        fill_layer(pkg, lib, h, LAYER, k, v)
    q = rng.standard_normal((16, 128), dtype=np.float32)
    kn = rng.standard_normal((8, 128), dtype=np.float32)
    vn = rng.standard_normal((8, 128), dtype=np.float32)
    return h, q, kn, vn


MODES = [("device", "device"), ("pinned", "pinned"), ("pageable", "pageable"), ("pinned", "device"),
         ("device", "pinned"), ("pageable", "pinned"), ("pinned", "pageable"), ("device", "pageable")]


def _append_call(pkg, lib, h, q, kn, vn, n, mode, heads=None):
    cs = pkg.cache_struct(h)
    cs.seq_len = n
    qb, qp = _buf(mode[0], q.shape, q)
    kb, kp = _buf(mode[0], kn.shape, kn)
    vb, vp_ = _buf(mode[0], vn.shape, vn)
    rows = 16 if heads is None else 2 * heads[1]
    ob, op = _buf(mode[1], (rows, 128))
    if heads is None:
        rc = lib.attention_decode_append_gqa(qp, kp, vp_, h, op, LAYER, SCALE)
    else:
        rc = lib.attention_decode_append_gqa_heads(qp, kp, vp_, h, op, LAYER, SCALE, heads[0], heads[1])
    assert rc == 0, pkg.last_error(lib)
    assert lib.attn_sync() == 0, pkg.last_error(lib)
    return _read(ob)


# kv_len 1 and 100: one split per head; 4,097: BF16 tensor-core splits (18 per head), FP32
# splits; 9,000: BF16 streaming spans
@pytest.mark.parametrize("dtype", [0, 1])
@pytest.mark.parametrize("kv_len", [1, 100, 4097, 9000])
def test_append_call_same_bits_for_every_residency(pkg, lib, dtype, kv_len):
    n = kv_len - 1
    h, q, kn, vn = _setup(pkg, lib, dtype, n, 100 + kv_len + dtype)
    try:
        ref = _append_call(pkg, lib, h, q, kn, vn, n, MODES[0])
        assert np.isfinite(ref).all()
        for mode in MODES[1:]:
            got = _append_call(pkg, lib, h, q, kn, vn, n, mode)
            assert np.array_equal(got, ref), f"{mode}: max diff {np.abs(got - ref).max()}"
    finally:
        lib.kv_cache_free(h)


@pytest.mark.parametrize("dtype", [0, 1])
@pytest.mark.parametrize("heads", [(2, 1), (4, 4), (0, 2)])
def test_head_subsets_same_bits(pkg, lib, dtype, heads):
    n = 6000
    h, q, kn, vn = _setup(pkg, lib, dtype, n, 7 + heads[0] + 10 * heads[1] + dtype)
    try:
        ref = _append_call(pkg, lib, h, q, kn, vn, n, ("device", "device"), heads)
        for mode in (("pinned", "pinned"), ("pageable", "pageable"), ("device", "pinned")):
            got = _append_call(pkg, lib, h, q, kn, vn, n, mode, heads)
            assert np.array_equal(got, ref), f"{mode}"
    finally:
        lib.kv_cache_free(h)


@pytest.mark.parametrize("dtype", [0, 1])
def test_plain_decode_and_deferred_append_same_bits(pkg, lib, dtype):
    n = 3000
    h, q, kn, vn = _setup(pkg, lib, dtype, n, 55 + dtype)
    cs = pkg.cache_struct(h)
    try:
        outs = {}
        for mode in MODES:
            qb, qp = _buf(mode[0], q.shape, q)
            ob, op = _buf(mode[1], (16, 128))
            lib.attention_decode_gqa(qp, h, op, LAYER, n, SCALE)
            pkg.check(lib, f"decode {mode}")
            assert lib.attn_sync() == 0
            outs[mode] = _read(ob)
        for mode in MODES[1:]:
            assert np.array_equal(outs[mode], outs[MODES[0]]), f"plain decode {mode}"
        # the deferred append of decoder.c: kv_cache_append from host rows, then the decode over
        # seq_len + 1 rows appends and attends in one launch
        ref = None
        for mode in (("device", "device"), ("pinned", "pinned"), ("pageable", "pageable"), ("pinned", "device")):
            cs.seq_len = n
            kr, vr = kn.copy(), vn.copy()
            lib.kv_cache_append(h, LAYER, vp(kr), vp(vr))
            qb, qp = _buf(mode[0], q.shape, q)
            ob, op = _buf(mode[1], (16, 128))
            lib.attention_decode_gqa(qp, h, op, LAYER, n + 1, SCALE)
            pkg.check(lib, f"deferred {mode}")
            assert lib.attn_sync() == 0
            got = _read(ob)
            if ref is None:
                ref = got
            assert np.array_equal(got, ref), f"deferred {mode}"
        assert np.array_equal(ref, _append_call(pkg, lib, h, q, kn, vn, n, ("device", "device")))
    finally:
        lib.kv_cache_free(h)


def test_back_to_back_calls_return_their_own_results(pkg, lib):
    """Calls on every third layer in turn with page-locked buffers, as a decode step makes them:
    each returns with its own layer's result in place (before any synchronisation), equal to the
    device-buffer call."""
    n = 2000
    rng = np.random.default_rng(9)
    h = new_cache(pkg, lib, n + 8, 1)
    cs = pkg.cache_struct(h)
    try:
        layers = list(range(0, 28, 3))
        for layer in layers:
            fill_layer(pkg, lib, h, layer, rng.standard_normal((n, 8, 128), dtype=np.float32),
                       rng.standard_normal((n, 8, 128), dtype=np.float32))
        qs = rng.standard_normal((len(layers), 16, 128), dtype=np.float32)
        kn = rng.standard_normal((8, 128), dtype=np.float32)
        vn = rng.standard_normal((8, 128), dtype=np.float32)
        cs.seq_len = n
        dq, dk, dv = (torch.from_numpy(x).cuda() for x in (qs, kn, vn))
        dout = torch.zeros((len(layers), 16, 128), device="cuda")
        for i, layer in enumerate(layers):
            rc = lib.attention_decode_append_gqa(ctypes.c_void_p(dq[i].data_ptr()), ctypes.c_void_p(dk.data_ptr()),
                                                 ctypes.c_void_p(dv.data_ptr()), h,
                                                 ctypes.c_void_p(dout[i].data_ptr()), layer, SCALE)
            assert rc == 0, pkg.last_error(lib)
        assert lib.attn_sync() == 0
        want = dout.cpu().numpy()
        pq = torch.from_numpy(qs).pin_memory()
        pk, pv = torch.from_numpy(kn).pin_memory(), torch.from_numpy(vn).pin_memory()
        po = torch.zeros((len(layers), 16, 128)).pin_memory()
        for rep in range(3):
            po.zero_()
            for i, layer in enumerate(layers):
                rc = lib.attention_decode_append_gqa(ctypes.c_void_p(pq[i].data_ptr()), ctypes.c_void_p(pk.data_ptr()),
                                                     ctypes.c_void_p(pv.data_ptr()), h,
                                                     ctypes.c_void_p(po[i].data_ptr()), layer, SCALE)
                assert rc == 0, pkg.last_error(lib)
                # the call returned: its output is there, before any synchronisation
                assert np.array_equal(po[i].numpy(), want[i]), f"rep {rep} layer {layer}"
    finally:
        lib.kv_cache_free(h)
