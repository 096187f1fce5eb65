"""KV-head sharding set up from C (attn_shard_init, include/attn_ext.h): the IPC handles go
through a caller-supplied all-gather callback, then attention_prefill_fused_gqa_sharded stores
every output row from the tensor-core epilogue into every rank's exchange buffer and
attention_decode_append_gqa_sharded gathers the decode output in the decode kernel.

* one rank on one GPU (the callback copies its own bytes): the assembled prefill output equals
  attention_prefill_fused_gqa bit for bit over three calls (both exchange slots); the decode
  equals attention_decode_append_gqa;
* two ranks on two GPUs (child processes, torch.distributed gloo behind the callback): each rank
  owns 4 KV heads, and every rank's assembled outputs equal the unsharded calls -- prefill bit for
  bit, decode to FP32 summation order (the split planner sees fewer heads)."""

import ctypes
import importlib
import os

import numpy as np
import pytest
import torch

from gpu_helpers import new_cache, vp

pytestmark = pytest.mark.gpu
SCALE = ctypes.c_float(0.08838834764831843)
EPS = ctypes.c_float(1e-6)
DEC_RTOL, DEC_ATOL = 1e-4, 1e-5


def _inputs(pkg, oracle, S, seed):
    wl = importlib.import_module(pkg.__name__ + ".workloads")
    rng = np.random.default_rng(seed)
    pos = wl.mrope_positions(4, 5, S - 20)
    q, k, v = wl.qkv(rng, S)
    qn, kn = wl.norm_weights(rng)
    cos, sin = oracle.mrope_cos_sin_3d(pos)
    dev = lambda a, dt=torch.float32: torch.from_numpy(np.ascontiguousarray(a)).to(dt).cuda()  # noqa: E731
    return [dev(q, torch.bfloat16), dev(k, torch.bfloat16), dev(v, torch.bfloat16), dev(qn), dev(kn), dev(cos),
            dev(sin)]


def _run_prefills_and_decode(pkg, lib, t, S, layers=(3, 4, 5)):
    """Sharded and unsharded prefill of `layers`, then one decode step of the last layer; returns
    (pairs of prefill outputs, pair of decode outputs)."""
    q, k, v, qn, kn, cos, sin = t
    ha = new_cache(pkg, lib, S + 4, pkg.ATTN_KV_BF16)
    hb = new_cache(pkg, lib, S + 4, pkg.ATTN_KV_BF16)
    pre, dec = [], None
    try:
        for layer in layers:
            full = torch.empty((S, 16, 128), dtype=torch.bfloat16, device="cuda")
            pkg.cache_struct(ha).seq_len = 0
            pkg.cache_struct(hb).seq_len = 0
            assert lib.attention_prefill_fused_gqa(vp(q), vp(k), vp(v), 1, vp(qn), vp(kn), vp(cos), vp(sin), ha, layer,
                                                   vp(full), 1, S, SCALE, EPS) == 0, pkg.last_error(lib)
            out = ctypes.c_void_p()
            assert lib.attention_prefill_fused_gqa_sharded(vp(q), vp(k), vp(v), 1, vp(qn), vp(kn), vp(cos), vp(sin),
                                                           hb, layer, S, SCALE, EPS, ctypes.byref(out)) == 0, \
                pkg.last_error(lib)
            assert lib.attn_sync() == 0, pkg.last_error(lib)
            got = _device_bf16(out.value, (S, 16, 128))
            pre.append((got, full))
        layer = layers[-1]
        pkg.cache_struct(ha).seq_len = S
        pkg.cache_struct(hb).seq_len = S
        qd = torch.randn((16, 128), device="cuda", generator=torch.Generator(device="cuda").manual_seed(5))
        kd = torch.randn((8, 128), device="cuda", generator=torch.Generator(device="cuda").manual_seed(6))
        vd = torch.randn((8, 128), device="cuda", generator=torch.Generator(device="cuda").manual_seed(7))
        want = torch.zeros((16, 128), device="cuda")
        got = torch.full((16, 128), float("nan"), device="cuda")
        assert lib.attention_decode_append_gqa(vp(qd), vp(kd), vp(vd), ha, vp(want), layer, SCALE) == 0
        assert lib.attention_decode_append_gqa_sharded(vp(qd), vp(kd), vp(vd), hb, vp(got), layer, SCALE) == 0, \
            pkg.last_error(lib)
        assert lib.attn_sync() == 0, pkg.last_error(lib)
        dec = (got, want)
    finally:
        torch.cuda.synchronize()
        lib.kv_cache_free(ha)
        lib.kv_cache_free(hb)
    return pre, dec


def _device_bf16(addr, shape):
    """A copy of the BF16 device tensor at `addr` (the library's exchange slot)."""
    n = int(np.prod(shape))
    out = torch.empty(shape, dtype=torch.bfloat16, device="cuda")
    cudart = ctypes.CDLL("libcudart.so.12")
    cudart.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
    assert cudart.cudaMemcpy(out.data_ptr(), addr, n * 2, 3) == 0  # device to device
    return out


def test_sharded_one_rank_equals_unsharded(pkg, lib, oracle):
    def own(send, recv, n, user):
        ctypes.memmove(recv, send, n)
        return 0
    cb = pkg.ALLGATHER_FN(own)
    S = 300
    assert lib.attn_shard_init(0, 1, S, ctypes.cast(cb, ctypes.c_void_p), None) == 0, pkg.last_error(lib)
    try:
        h0, n = ctypes.c_int(), ctypes.c_int()
        assert lib.attn_shard_heads(ctypes.byref(h0), ctypes.byref(n)) == 0 and (h0.value, n.value) == (0, 8)
        t = _inputs(pkg, oracle, S, 11)
        pre, (got, want) = _run_prefills_and_decode(pkg, lib, t, S)
        for a, b in pre:
            assert torch.equal(a, b)
        assert torch.equal(got, want)
        # beyond max_tokens: refused
        out = ctypes.c_void_p()
        hx = new_cache(pkg, lib, S + 8, pkg.ATTN_KV_BF16)
        try:
            lib.attn_clear_error()
            rc = lib.attention_prefill_fused_gqa_sharded(vp(t[0]), vp(t[1]), vp(t[2]), 1, vp(t[3]), vp(t[4]),
                                                         vp(t[5]), vp(t[6]), hx, 0, S + 1, SCALE, EPS,
                                                         ctypes.byref(out))
            assert rc != 0 and "max_tokens" in pkg.last_error(lib)
            lib.attn_clear_error()
        finally:
            lib.kv_cache_free(hx)
    finally:
        lib.attn_shard_close()


def _two_rank_worker(rank, world, port, result_dir):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    import datetime

    import torch.distributed as dist
    from gpu_helpers import load_pkg_and_lib

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    pkg, lib = load_pkg_and_lib()
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
    import oracle as orc
    shard = importlib.import_module(pkg.__name__ + ".shard")
    S = 700
    grp = shard.ShardGroup(lib, max_tokens=S)
    ok = (grp.kv_head0, grp.kv_heads) == (4 * rank, 4)
    try:
        t = _inputs(pkg, orc.Oracle(), S, 21)  # the same inputs on every rank
        pre, (got, want) = _run_prefills_and_decode(pkg, lib, t, S)
        ok = ok and all(bool(torch.equal(a, b)) for a, b in pre)
        ok = ok and bool(torch.isfinite(got).all()) and torch.allclose(got, want, rtol=DEC_RTOL, atol=DEC_ATOL)
    finally:
        torch.cuda.synchronize()
        dist.barrier()
        grp.close()
        dist.destroy_process_group()
    with open(os.path.join(result_dir, f"rank{rank}"), "w") as f:
        f.write("ok" if ok else "mismatch")


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sharded_two_ranks_equal_unsharded(tmp_path):
    import socket
    import time

    import torch.multiprocessing as mp
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        port = sock.getsockname()[1]
    ctx = mp.start_processes(_two_rank_worker, args=(2, port, str(tmp_path)), nprocs=2, join=False,
                             start_method="spawn")
    deadline = time.time() + 300
    while not ctx.join(timeout=10):
        assert time.time() < deadline, "ranks did not finish"
    for r in range(2):
        assert (tmp_path / f"rank{r}").read_text() == "ok", r
