"""KV-head sharding of one long sequence, host logic on CPU: two `gloo`
ranks each compute their KV heads' attention (the oracle, with the other heads' K/V zeroed --
heads are independent), all-gather the head-major shards in rank order and restore the
token-major layout; the result must equal the unsharded attention exactly."""

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, result_dir):
    import torch
    import torch.distributed as dist

    sys.path.insert(0, str(ROOT / "tests"))
    sys.path.insert(0, str(ROOT / "oracle"))
    from conftest import load_pkg
    import oracle as orc

    pkg = load_pkg()
    shard = __import__(pkg.__name__ + ".shard", fromlist=["shard"])
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        o = orc.Oracle()
        rng = np.random.default_rng(11)
        S = 37
        q = rng.standard_normal((S, 16, 128), dtype=np.float32)
        k = rng.standard_normal((S, 8, 128), dtype=np.float32)
        v = rng.standard_normal((S, 8, 128), dtype=np.float32)
        h0, n = shard.kv_head_range(rank, world)
        q0, nq = shard.query_head_range(rank, world)
        # Only this rank's heads carry data: the other heads' K/V are zero.
        kk, vv = np.zeros_like(k), np.zeros_like(v)
        kk[:, h0:h0 + n], vv[:, h0:h0 + n] = k[:, h0:h0 + n], v[:, h0:h0 + n]
        mine = o.prefill(q, kk, vv)[:, q0:q0 + nq]               # [S][nq][128]
        part = torch.from_numpy(np.ascontiguousarray(mine.swapaxes(0, 1)))  # head-major shard
        full = shard.gather_heads(part)                          # [16][S][128]
        got = shard.tokens_from_heads(full).numpy()
        want = o.prefill(q, k, v)
        np.save(os.path.join(result_dir, f"r{rank}.npy"), np.array([float(np.max(np.abs(got - want)))]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_shard_gather_matches_unsharded(world, tmp_path):
    import torch.multiprocessing as mp

    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(world):
        assert np.load(tmp_path / f"r{r}.npy")[0] == 0.0


def test_head_ranges(pkg):
    shard = __import__(pkg.__name__ + ".shard", fromlist=["shard"])
    for world in (1, 2, 4, 8):
        heads = [h for r in range(world) for h in range(*(lambda a, n: (a, a + n))(*shard.kv_head_range(r, world)))]
        assert heads == list(range(8))
        assert shard.query_head_range(world - 1, world)[0] + shard.query_head_range(world - 1, world)[1] == 16
    with pytest.raises(ValueError):
        shard.kv_head_range(0, 3)
    with pytest.raises(ValueError):
        shard.kv_head_range(2, 2)
