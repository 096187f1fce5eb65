"""KV-head shards through the C-ABI on one GPU: the shards of every rank count (2, 4, 8),
gathered head-major and relaid token-major by attn_heads_to_tokens, must equal the unsharded
entry points -- bit for bit for prefill (the same tiles compute each head either way); for
decode to FP32 summation order, since fewer heads per launch let the planner pick shorter
splits (tolerance DEC_RTOL / DEC_ATOL, written here)."""

import ctypes
import importlib

import numpy as np
import pytest
import torch

from gpu_helpers import new_cache, vp

pytestmark = pytest.mark.gpu
SCALE = ctypes.c_float(0.08838834764831843)
DEC_RTOL, DEC_ATOL = 1e-4, 1e-5
EPS = ctypes.c_float(1e-6)


def _prefill_inputs(pkg, oracle, S, seed):
    wl = importlib.import_module(pkg.__name__ + ".workloads")
    rng = np.random.default_rng(seed)
    pos = wl.mrope_positions(4, 5, S - 20)
    q, k, v = wl.qkv(rng, S)
    qn, kn = wl.norm_weights(rng)
    cos, sin = oracle.mrope_cos_sin_3d(pos)
    dev = lambda a, dt=torch.float32: torch.from_numpy(np.ascontiguousarray(a)).to(dt).cuda()
    return dev(q, torch.bfloat16), dev(k, torch.bfloat16), dev(v, torch.bfloat16), dev(qn), dev(kn), dev(cos), dev(sin)


@pytest.mark.parametrize("S,off", [(300, 0), (129, 200)])
def test_prefill_shards_equal_unsharded(pkg, lib, oracle, S, off):
    shard = importlib.import_module(pkg.__name__ + ".shard")
    q, k, v, qn, kn, cos, sin = _prefill_inputs(pkg, oracle, S, 3 + S)
    rows = off + S + 2
    full = torch.empty((S, 16, 128), dtype=torch.bfloat16, device="cuda")
    h = new_cache(pkg, lib, rows, pkg.ATTN_KV_BF16)
    try:
        if off:
            old = torch.randn((off, 8, 128), device="cuda")
            lib.kv_cache_append_prefill(h, 5, vp(old), vp(old), off)
        pkg.cache_struct(h).seq_len = off
        rc = lib.attention_prefill_fused_gqa(vp(q), vp(k), vp(v), pkg.ATTN_DT_BF16, vp(qn), vp(kn), vp(cos), vp(sin),
                                             h, 5, vp(full), pkg.ATTN_DT_BF16, S, SCALE, EPS)
        assert rc == 0, pkg.last_error(lib)
        for world in (2, 4, 8):
            parts = []
            for r in range(world):
                h0, n = shard.kv_head_range(r, world)
                part = torch.empty((2 * n, S, 128), dtype=torch.bfloat16, device="cuda")
                rc = lib.attention_prefill_fused_gqa_heads(vp(q), vp(k), vp(v), pkg.ATTN_DT_BF16, vp(qn), vp(kn),
                                                           vp(cos), vp(sin), h, 5, vp(part), pkg.ATTN_DT_BF16, S,
                                                           SCALE, EPS, h0, n)
                assert rc == 0, pkg.last_error(lib)
                parts.append(part)
            gathered = torch.cat(parts, 0).contiguous()
            tokens = torch.empty_like(full)
            assert lib.attn_heads_to_tokens(vp(gathered), vp(tokens), S, pkg.ATTN_DT_BF16) == 0, pkg.last_error(lib)
            assert lib.attn_sync() == 0, pkg.last_error(lib)
            assert torch.equal(tokens, full), world
    finally:
        lib.kv_cache_free(h)


# 20,000 and 33,000 rows: a head's splits merged by one CTA from L2 (8 heads), through shared
# memory (33-64 records: 4 heads) and in two levels (more than 64: 1 and 2 heads)
@pytest.mark.parametrize("kv_len", [1, 700, 4097, 20000, 33000])
def test_decode_shards_equal_unsharded(pkg, lib, kv_len):
    shard = importlib.import_module(pkg.__name__ + ".shard")
    pos = kv_len - 1
    h = new_cache(pkg, lib, kv_len + 3, pkg.ATTN_KV_BF16)
    try:
        if pos:
            old = torch.randn((pos, 8, 128), device="cuda")
            lib.kv_cache_append_prefill(h, 2, vp(old), vp(old), pos)
        pkg.cache_struct(h).seq_len = pos
        q = torch.randn((16, 128), device="cuda")
        kn, vn = torch.randn((8, 128), device="cuda"), torch.randn((8, 128), device="cuda")
        full = torch.empty((16, 128), device="cuda")
        assert lib.attention_decode_append_gqa(vp(q), vp(kn), vp(vn), h, vp(full), 2, SCALE) == 0, pkg.last_error(lib)
        for world in (2, 4, 8):
            out = torch.full((16, 128), float("nan"), device="cuda")
            for r in range(world):
                h0, n = shard.kv_head_range(r, world)
                q0, _ = shard.query_head_range(r, world)
                rc = lib.attention_decode_append_gqa_heads(vp(q), vp(kn), vp(vn), h, vp(out[q0]), 2, SCALE, h0, n)
                assert rc == 0, pkg.last_error(lib)
            assert lib.attn_sync() == 0, pkg.last_error(lib)
            assert torch.allclose(out, full, rtol=DEC_RTOL, atol=DEC_ATOL), (world, (out - full).abs().max().item())
    finally:
        lib.kv_cache_free(h)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_heads_to_tokens(pkg, lib, dtype):
    tdt = torch.float32 if dtype == "f32" else torch.bfloat16
    src = torch.randn((16, 77, 128), device="cuda").to(tdt)
    dst = torch.empty((77, 16, 128), device="cuda", dtype=tdt)
    code = pkg.ATTN_DT_F32 if dtype == "f32" else pkg.ATTN_DT_BF16
    assert lib.attn_heads_to_tokens(vp(src), vp(dst), 77, code) == 0, pkg.last_error(lib)
    assert lib.attn_sync() == 0
    assert torch.equal(dst, src.transpose(0, 1))


def test_shard_rejects_bad_heads(pkg, lib):
    h = new_cache(pkg, lib, 8, pkg.ATTN_KV_BF16)
    x = torch.zeros((16, 128), device="cuda")
    try:
        for h0, n in ((0, 0), (7, 2), (-1, 1), (0, 9)):
            lib.attn_clear_error()
            rc = lib.attention_decode_append_gqa_heads(vp(x), vp(x), vp(x), h, vp(x), 0, SCALE, h0, n)
            assert rc != 0 and "KV heads" in pkg.last_error(lib)
    finally:
        lib.attn_clear_error()
        lib.kv_cache_free(h)
