"""KV-head sharding of one long sequence over N GPUs (one process per GPU).

GQA heads are independent: KV head h and its query heads 2h, 2h+1 need nothing from the other
heads, so a single long sequence is split by KV head, 8/N heads per rank.
Each rank appends its heads' K/V rows to its own cache and computes its query heads' attention
as one contiguous head-major shard [2*(8/N)][S][128] (attention_prefill_fused_gqa_heads /
attention_decode_append_gqa_heads); one all-gather in rank order assembles [16][S][128], and
attn_heads_to_tokens (or tokens_from_heads, for host tensors) restores the token-major
[S][16][128] layout the reference's decoder.c consumes.  The reference itself runs on one
CPU and has no such path.
"""

from __future__ import annotations

KV_HEADS = 8
Q_PER_KV = 2


def kv_head_range(rank: int, world: int) -> tuple[int, int]:
    """(first KV head, number of KV heads) owned by `rank` of `world` ranks; world must
    divide the 8 KV heads (1, 2, 4 or 8)."""
    if world < 1 or KV_HEADS % world:
        raise ValueError(f"world size {world} does not divide the {KV_HEADS} KV heads")
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside [0, {world})")
    n = KV_HEADS // world
    return rank * n, n


def query_head_range(rank: int, world: int) -> tuple[int, int]:
    """(first query head, number of query heads) whose outputs `rank` produces."""
    h0, n = kv_head_range(rank, world)
    return Q_PER_KV * h0, Q_PER_KV * n


def gather_heads(shard, group=None):
    """All-gather the head-major shards [2n][S][128] of every rank, in rank order, into
    [16][S][128] (torch tensors; NCCL for CUDA tensors, any backend for host ones)."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    out = shard.new_empty((shard.shape[0] * world,) + tuple(shard.shape[1:]))
    if shard.is_cuda:
        dist.all_gather_into_tensor(out, shard.contiguous(), group=group)
    else:
        parts = list(out.chunk(world, dim=0))
        dist.all_gather(parts, shard.contiguous(), group=group)
        out = torch.cat(parts, dim=0)
    return out


def tokens_from_heads(gathered):
    """Head-major [16][S][128] -> token-major [S][16][128] (host-side twin of
    attn_heads_to_tokens, for tensors or arrays)."""
    return gathered.swapaxes(0, 1)


class PeerGather:
    """The library's decode output gather over NVLink (attn_gather_*), set up for the ranks of
    `group`: each rank allocates its exchange buffer, the 64-byte CUDA IPC handles are
    exchanged with torch.distributed (any backend) and the peers' buffers mapped.  Then
    attention_decode_append_gqa_gathered returns the whole [16][128] output on every rank.
    close() after the last call (all of them completed)."""

    def __init__(self, lib, group=None):
        import ctypes
        import torch.distributed as dist

        self.lib = lib
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        if lib.attn_gather_init(rank, world):
            raise RuntimeError((lib.attn_last_error() or b"").decode())
        try:
            h = (ctypes.c_char * 64)()
            if lib.attn_gather_handle(h):
                raise RuntimeError((lib.attn_last_error() or b"").decode())
            handles = [None] * world
            dist.all_gather_object(handles, bytes(h), group=group)
            blob = b"".join(handles)
            buf = (ctypes.c_char * len(blob)).from_buffer_copy(blob)
            if lib.attn_gather_connect(buf):
                raise RuntimeError((lib.attn_last_error() or b"").decode())
        except BaseException:
            lib.attn_gather_close()
            raise

    def close(self):
        if self.lib is not None:
            self.lib.attn_gather_close()
            self.lib = None


class ShardGroup:
    """attn_shard_init for the ranks of a torch.distributed group: the library's all-gather
    callback is served by torch.distributed (any backend; host bytes).  Afterwards
    attention_prefill_fused_gqa_sharded / attention_decode_append_gqa_sharded run this rank's KV
    heads and leave the whole output on every rank, with no collective call.  close() after the
    last call has completed.  (A C caller passes its own callback -- MPI, a TCP store, ...)"""

    def __init__(self, lib, max_tokens, group=None):
        import ctypes

        import torch.distributed as dist

        self.lib = lib
        self.group = group
        rank, world = dist.get_rank(group), dist.get_world_size(group)

        def allgather(send, recv, nbytes, user):
            try:
                mine = ctypes.string_at(send, nbytes)
                parts = [None] * world
                dist.all_gather_object(parts, mine, group=group)
                blob = b"".join(parts)
                ctypes.memmove(recv, blob, len(blob))
                return 0
            except Exception:  # noqa: BLE001 -- reported to the library as a failed exchange
                return 1

        pkg = __import__(__name__.rsplit(".", 1)[0])
        self._cb = pkg.ALLGATHER_FN(allgather)  # kept alive while the library may call it
        if lib.attn_shard_init(rank, world, int(max_tokens), ctypes.cast(self._cb, ctypes.c_void_p), None):
            raise RuntimeError((lib.attn_last_error() or b"").decode())
        h0, n = ctypes.c_int(), ctypes.c_int()
        lib.attn_shard_heads(ctypes.byref(h0), ctypes.byref(n))
        self.kv_head0, self.kv_heads = h0.value, n.value

    def close(self):
        if self.lib is not None:
            self.lib.attn_shard_close()
            self.lib = None
