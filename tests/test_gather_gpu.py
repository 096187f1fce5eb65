"""Decode output gather over NVLink (attention_decode_append_gqa_gathered): one rank (the
protocol on one GPU, against the unsharded call, eager and replayed from a CUDA graph) and,
where two GPUs are visible, two ranks in child processes against the unsharded decode."""

import ctypes
import os

import numpy as np
import pytest
import torch

from gpu_helpers import fill_layer, new_cache, vp

pytestmark = pytest.mark.gpu
SCALE = ctypes.c_float(0.08838834764831843)


def _single_rank_gather(lib):
    h = (ctypes.c_char * 64)()
    assert lib.attn_gather_init(0, 1) == 0
    assert lib.attn_gather_handle(h) == 0
    assert lib.attn_gather_connect(h) == 0


def test_gather_one_rank_matches_plain_decode(pkg, lib):
    rng = np.random.default_rng(77)
    n = 4500
    k = rng.standard_normal((n + 8, 8, 128), dtype=np.float32)
    v = rng.standard_normal((n + 8, 8, 128), dtype=np.float32)
    ha = new_cache(pkg, lib, n + 8, pkg.ATTN_KV_BF16)
    hb = new_cache(pkg, lib, n + 8, pkg.ATTN_KV_BF16)
    _single_rank_gather(lib)
    try:
        fill_layer(pkg, lib, ha, 3, k[:n], v[:n])
        fill_layer(pkg, lib, hb, 3, k[:n], v[:n])
        for step in range(5):  # both exchange slots, several epochs
            pkg.cache_struct(ha).seq_len = n + step
            pkg.cache_struct(hb).seq_len = n + step
            q = torch.tensor(rng.standard_normal((16, 128), dtype=np.float32), device="cuda")
            kn = torch.tensor(k[n + step], device="cuda")
            vn = torch.tensor(v[n + step], device="cuda")
            want = torch.zeros((16, 128), device="cuda")
            got = torch.full((16, 128), float("nan"), device="cuda")
            assert lib.attention_decode_append_gqa(vp(q), vp(kn), vp(vn), ha, vp(want), 3, SCALE) == 0
            assert lib.attention_decode_append_gqa_gathered(vp(q), vp(kn), vp(vn), hb, vp(got), 3, SCALE, 0, 8) == 0
            assert lib.attn_sync() == 0, pkg.last_error(lib)
            assert torch.equal(got, want), step
        # replayed from a CUDA graph: the epochs advance on the device
        s = torch.cuda.Stream()
        lib.attn_set_stream(ctypes.c_void_p(s.cuda_stream))
        pkg.cache_struct(hb).seq_len = n + 5
        q = torch.randn((16, 128), device="cuda")
        kn, vn = torch.randn((8, 128), device="cuda"), torch.randn((8, 128), device="cuda")
        got = torch.zeros((16, 128), device="cuda")
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            assert lib.attention_decode_append_gqa_gathered(vp(q), vp(kn), vp(vn), hb, vp(got), 3, SCALE, 0, 8) == 0
        outs = []
        for _ in range(3):
            got.zero_()
            g.replay()
            s.synchronize()
            outs.append(got.clone())
        lib.attn_set_stream(None)
        assert lib.attn_sync() == 0, pkg.last_error(lib)
        pkg.cache_struct(ha).seq_len = n + 5
        want = torch.zeros((16, 128), device="cuda")
        assert lib.attention_decode_append_gqa(vp(q), vp(kn), vp(vn), ha, vp(want), 3, SCALE) == 0
        torch.cuda.synchronize()
        for o in outs:
            assert torch.equal(o, want)
        del g
    finally:
        torch.cuda.synchronize()
        lib.attn_gather_close()
        lib.kv_cache_free(ha)
        lib.kv_cache_free(hb)


def test_gathered_requires_setup(pkg, lib):
    h = new_cache(pkg, lib, 64, pkg.ATTN_KV_BF16)
    try:
        q = torch.zeros((16, 128), device="cuda")
        kn = torch.zeros((8, 128), device="cuda")
        lib.attn_clear_error()
        rc = lib.attention_decode_append_gqa_gathered(vp(q), vp(kn), vp(kn), h, vp(q), 0, SCALE, 0, 8)
        assert rc != 0 and "gather" in pkg.last_error(lib)
        lib.attn_clear_error()
    finally:
        lib.kv_cache_free(h)


def _two_rank_worker(rank, world, port, result_dir):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    import datetime

    import torch.distributed as dist
    from gpu_helpers import fill_layer as fill, load_pkg_and_lib, new_cache as newc, vp as vptr

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    pkg, lib = load_pkg_and_lib()
    shard = __import__(pkg.__name__ + ".shard", fromlist=["PeerGather"])
    rng = np.random.default_rng(99)
    n = 6000
    k = rng.standard_normal((n + 4, 8, 128), dtype=np.float32)
    v = rng.standard_normal((n + 4, 8, 128), dtype=np.float32)
    qs = rng.standard_normal((3, 16, 128), dtype=np.float32)
    ha = newc(pkg, lib, n + 4, pkg.ATTN_KV_BF16)
    hb = newc(pkg, lib, n + 4, pkg.ATTN_KV_BF16)
    pg = shard.PeerGather(lib)
    h0, nh = shard.kv_head_range(rank, world)
    ok = True
    try:
        fill(pkg, lib, ha, 1, k[:n], v[:n])
        fill(pkg, lib, hb, 1, k[:n], v[:n])
        for step in range(3):
            pkg.cache_struct(ha).seq_len = n + step
            pkg.cache_struct(hb).seq_len = n + step
            q = torch.tensor(qs[step], device="cuda")
            kn, vn = torch.tensor(k[n + step], device="cuda"), torch.tensor(v[n + step], device="cuda")
            want = torch.zeros((16, 128), device="cuda")
            got = torch.full((16, 128), float("nan"), device="cuda")
            assert lib.attention_decode_append_gqa(vptr(q), vptr(kn), vptr(vn), ha, vptr(want), 1, SCALE) == 0
            rc = lib.attention_decode_append_gqa_gathered(vptr(q), vptr(kn), vptr(vn), hb, vptr(got), 1, SCALE, h0, nh)
            assert rc == 0, pkg.last_error(lib)
            assert lib.attn_sync() == 0, pkg.last_error(lib)
            ok = ok and bool(torch.isfinite(got).all()) and torch.allclose(got, want, rtol=1e-4, atol=1e-5)
    finally:
        torch.cuda.synchronize()
        dist.barrier()
        pg.close()
        lib.kv_cache_free(ha)
        lib.kv_cache_free(hb)
        dist.destroy_process_group()
    with open(os.path.join(result_dir, f"rank{rank}"), "w") as f:
        f.write("ok" if ok else "mismatch")


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_gather_two_ranks(tmp_path):
    import socket

    import torch.multiprocessing as mp
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        port = sock.getsockname()[1]
    import time
    ctx = mp.start_processes(_two_rank_worker, args=(2, port, str(tmp_path)), nprocs=2, join=False,
                             start_method="spawn")
    deadline = time.time() + 300
    while not ctx.join(timeout=10):  # True once every process has exited (raises if one failed)
        assert time.time() < deadline, "ranks did not finish"

    for r in range(2):
        assert (tmp_path / f"rank{r}").read_text() == "ok", r
