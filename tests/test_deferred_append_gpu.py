"""kv_cache_append of one row from host memory, as kernel/decoder.c:96-100 issues it every decode
step, is deferred: the row is copied into the cache's page-locked slot for its layer at once (the
caller may reuse its buffers on return, as after the reference's memcpy), and written by the next
launch that touches the layer -- attention_decode_gqa over seq_len + 1 rows appends and attends
in one kernel.  Every other path that reads or writes the layer writes the row first.  Checked
here: the row reaches the cache on every path, and attention results match the oracle."""

import ctypes

import numpy as np
import pytest
import torch

from gpu_helpers import TOL_MAX, TOL_REL, d2h, fill_layer, head_first, new_cache, vp
from oracle import max_abs, rel_l2

pytestmark = pytest.mark.gpu
SCALE = ctypes.c_float(0.08838834764831843)
LAYER = 4


def _rows(rng, n):
    return (rng.standard_normal((n, 8, 128), dtype=np.float32), rng.standard_normal((n, 8, 128), dtype=np.float32))


@pytest.mark.parametrize("dtype", [0, 1])
def test_deferred_row_reaches_the_cache_on_every_path(pkg, lib, dtype):
    rng = np.random.default_rng(21 + dtype)
    n = 300
    k, v = _rows(rng, n + 4)
    h = new_cache(pkg, lib, n + 8, dtype)
    cs = pkg.cache_struct(h)
    try:
        fill_layer(pkg, lib, h, LAYER, k[:n], v[:n])
        cs.seq_len = n
        # 1) read back through kv_cache_k / kv_cache_v
        kr, vr = k[n].copy(), v[n].copy()
        lib.kv_cache_append(h, LAYER, vp(kr), vp(vr))
        pkg.check(lib, "append")
        kr[:] = 7.0  # the caller's buffer is free again on return
        vr[:] = 7.0
        el = np.uint16 if dtype else np.float32
        got_k = d2h(lib.kv_cache_k(h, LAYER, 0), (8, n + 8, 128), el)
        got_v = d2h(lib.kv_cache_v(h, LAYER, 0), (8, n + 8, 128), el)
        as_f32 = (lambda u: (u.astype(np.uint32) << 16).view(np.float32)) if dtype else (lambda x: x)
        tol = 2.0 ** -8 if dtype else 0.0
        assert np.allclose(as_f32(got_k)[:, n], k[n], rtol=tol, atol=0) and np.allclose(as_f32(got_v)[:, n], v[n], rtol=tol, atol=0)
        # 2) a second append to the same layer writes the first one's row before staging its own
        k1, v1, k2, v2 = k[n + 1].copy(), v[n + 1].copy(), k[n + 2].copy(), v[n + 2].copy()
        cs.seq_len = n + 1
        lib.kv_cache_append(h, LAYER, vp(k1), vp(v1))
        cs.seq_len = n + 2
        lib.kv_cache_append(h, LAYER, vp(k2), vp(v2))
        pkg.check(lib, "appends")
        # 3) attention over fewer rows than seq_len + 1: the row is written, then a plain decode
        q = rng.standard_normal((16, 128), dtype=np.float32)
        out = np.zeros((16, 128), dtype=np.float32)
        lib.attention_decode_gqa(vp(q), h, vp(out), LAYER, n + 2, SCALE)
        pkg.check(lib, "decode")
        got_k = as_f32(d2h(lib.kv_cache_k(h, LAYER, 0), (8, n + 8, 128), el))
        for r in (n + 1, n + 2):
            assert np.allclose(got_k[:, r], k[r], rtol=tol, atol=0), r
    finally:
        lib.kv_cache_free(h)


@pytest.mark.parametrize("dtype", [0, 1])
def test_append_then_decode_in_one_launch_matches_oracle(pkg, lib, oracle, dtype):
    """The decoder.c pair over several steps and layers: host q/k/v/output, FP32 and BF16 caches,
    device output buffers too (the call then only queues its work)."""
    rng = np.random.default_rng(40 + dtype)
    n0, steps = 1000, 6
    k, v = _rows(rng, n0 + steps)
    h = new_cache(pkg, lib, n0 + steps + 2, dtype)
    cs = pkg.cache_struct(h)
    bf = (lambda a: torch.from_numpy(np.ascontiguousarray(a)).bfloat16().float().numpy()) if dtype else (lambda a: a)
    try:
        for layer in (0, 27):
            fill_layer(pkg, lib, h, layer, k[:n0], v[:n0])
        cs.seq_len = n0
        for i in range(steps):
            qs = rng.standard_normal((2, 16, 128), dtype=np.float32)
            outs = []
            for j, layer in enumerate((0, 27)):
                kn, vn = k[n0 + i].copy(), v[n0 + i].copy()
                lib.kv_cache_append(h, layer, vp(kn), vp(vn))
                if j == 0:
                    out = np.zeros((16, 128), dtype=np.float32)
                    lib.attention_decode_gqa(vp(qs[j]), h, vp(out), layer, cs.seq_len + 1, SCALE)
                else:  # device query and output: queued, no wait
                    qd = torch.from_numpy(qs[j]).cuda()
                    od = torch.full((16, 128), float("nan"), device="cuda")
                    lib.attention_decode_gqa(vp(qd), h, vp(od), layer, cs.seq_len + 1, SCALE)
                    kn[:] = 0.0  # the caller's row buffer is free once the append returned
                    assert lib.attn_sync() == 0, pkg.last_error(lib)
                    out = od.cpu().numpy()
                pkg.check(lib, f"step {i} layer {layer}")
                outs.append(out)
            lib.kv_cache_advance(h, 1)
            for j in range(2):
                want = oracle.decode(qs[j], head_first(bf(k[:n0 + i + 1])), head_first(bf(v[:n0 + i + 1])), n0 + i + 1)
                assert max_abs(outs[j], want) <= TOL_MAX and rel_l2(outs[j], want) <= TOL_REL, (i, j)
    finally:
        lib.kv_cache_free(h)
