"""attention_decode_gqa_noalloc: the decode entry point for callers that cannot allocate
device memory (their memory belongs to another allocator's pool, or their footprint is
fixed), checked against the regular entry point attention_decode_gqa.

The file name makes pytest collect it last, so a run that stops at the first failure has
already run every other test.  It passes alone in a fresh process and after the others.
"""

import ctypes

import numpy as np
import pytest
import torch

from gpu_helpers import TOL_MAX, TOL_REL, check, dev, fill_layer, new_cache, vp
from oracle import max_abs, rel_l2

pytestmark = pytest.mark.gpu
SCALE = ctypes.c_float(0.08838834764831843)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_no_alloc_decode_matches_regular_entry_point(pkg, lib, dtype):
    kv_dt = pkg.ATTN_KV_F32 if dtype == "f32" else pkg.ATTN_KV_BF16
    rng = np.random.default_rng(2024)
    max_seq = 5000
    layer = 6
    k = rng.standard_normal((max_seq, 8, 128), dtype=np.float32)
    v = rng.standard_normal((max_seq, 8, 128), dtype=np.float32)
    h = new_cache(pkg, lib, max_seq, kv_dt)
    try:
        fill_layer(pkg, lib, h, layer, k, v)
        k_rows = lib.kv_cache_k(h, layer, 0)
        v_rows = lib.kv_cache_v(h, layer, 0)
        # Two calls in a row on the shared fixed scratch: a long one (many splits, merge
        # through the scratch records) and a different, shorter one.
        for kv_len in (4999, 1234):
            q = dev(rng.standard_normal((16, 128), dtype=np.float32))
            want = torch.zeros((16, 128), dtype=torch.float32, device="cuda")
            got = torch.full((16, 128), float("nan"), dtype=torch.float32, device="cuda")
            lib.attention_decode_gqa(vp(q), h, vp(want), layer, kv_len, SCALE)
            check(pkg, lib, "regular decode")
            rc = lib.attention_decode_gqa_noalloc(vp(q), k_rows, v_rows, max_seq, kv_dt, vp(got), kv_len,
                                                  SCALE, None)
            assert rc == 0, pkg.last_error(lib)
            torch.cuda.synchronize()
            assert lib.attn_sync() == 0, pkg.last_error(lib)
            w, g = want.cpu().numpy(), got.cpu().numpy()
            assert np.isfinite(g).all()
            assert max_abs(g, w) <= TOL_MAX and rel_l2(g, w) <= TOL_REL, kv_len
    finally:
        lib.kv_cache_free(h)


def test_no_alloc_decode_rejects_what_it_cannot_hold(pkg, lib):
    h = new_cache(pkg, lib, 30000, pkg.ATTN_KV_F32)
    try:
        k_rows = lib.kv_cache_k(h, 0, 0)
        v_rows = lib.kv_cache_v(h, 0, 0)
        q = torch.zeros((16, 128), dtype=torch.float32, device="cuda")
        out = torch.zeros_like(q)
        lib.attn_clear_error()
        rc = lib.attention_decode_gqa_noalloc(vp(q), k_rows, v_rows, 30000, pkg.ATTN_KV_F32, vp(out), 30000,
                                              SCALE, None)
        assert rc != 0 and "splits" in pkg.last_error(lib)
        lib.attn_clear_error()
        host_q = np.zeros((16, 128), dtype=np.float32)
        rc = lib.attention_decode_gqa_noalloc(vp(host_q), k_rows, v_rows, 30000, pkg.ATTN_KV_F32, vp(out), 10,
                                              SCALE, None)
        assert rc != 0 and "device memory" in pkg.last_error(lib)
        lib.attn_clear_error()
    finally:
        lib.kv_cache_free(h)
