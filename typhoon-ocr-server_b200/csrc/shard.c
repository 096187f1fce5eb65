/*
 * shard.c -- KV-head sharding of one long sequence over the GPUs of one node, set up and driven
 * from C (the reference runs on one CPU and has no multi-GPU path; this extends its attention
 * entry points the way the long-context configuration needs).
 *
 * One process (rank) per GPU.  attn_shard_init allocates this rank's two exchange buffers on the
 * current device -- the decode output exchange of decode.cu and the prefill output exchange of
 * prefill_tc.cu (tyb_prefill_x: a flag header, then two token-major [max_tokens][16][128] BF16
 * slots) -- and maps every peer's through CUDA IPC.  The 2 x 64-byte IPC handles of each rank are
 * exchanged through a caller-supplied all-gather callback, so any transport the caller already
 * has (MPI, a TCP store, NCCL over a host-staged buffer, torch.distributed) will do and the
 * library links no collective library.  After that, no collective call is needed: the kernels
 * store their outputs into every rank's buffer over NVLink -- the prefill raising a flag per
 * rank once its tiles are stored, the decode sending values that carry the call's number.
 */
#include <cuda_runtime_api.h>
#include <stdlib.h>
#include <string.h>

#include "attn_ext.h"
#include "host_internal.h"

#define TYB_IPC_HANDLE_BYTES 64

static struct {
    int active;
    int rank, nranks, max_tokens;
    void *px;                /* this rank's prefill exchange buffer (device) */
    void *peer_px[8];        /* every rank's, mapped (own at `rank`) */
    tyb_prefill_x *px_dev;   /* device copy of the table */
    /* the TMA maps of every rank's slots the prefill stores its output tiles through */
    unsigned char px_maps[TYB_PX_MAPS_BYTES] __attribute__((aligned(64)));
    unsigned int px_epoch;   /* sharded prefill calls made (host count; the kernel gets it) */
} g_sh;

static void shard_release(void)
{
    cudaDeviceSynchronize(); /* nothing may still touch the buffers */
    for (int p = 0; p < 8; p++) {
        if (g_sh.peer_px[p] && p != g_sh.rank) cudaIpcCloseMemHandle(g_sh.peer_px[p]);
        g_sh.peer_px[p] = NULL;
    }
    if (g_sh.px) cudaFree(g_sh.px);
    if (g_sh.px_dev) cudaFree(g_sh.px_dev);
    g_sh.px = NULL;
    g_sh.px_dev = NULL;
    tyb_gather_close();
    g_sh.active = 0;
    g_sh.px_epoch = 0;
}

int attn_shard_init(int rank, int nranks, int max_tokens, attn_allgather_fn allgather, void *user)
{
    const char *what = "attn_shard_init";
    if (nranks != 1 && nranks != 2 && nranks != 4 && nranks != 8) {
        tyb_set_error("%s: nranks %d does not divide the 8 KV heads (1, 2, 4 or 8)", what, nranks);
        return 1;
    }
    if (rank < 0 || rank >= nranks || max_tokens < 0 || max_tokens > TYB_MAX_SEQ || !allgather) {
        tyb_set_error("%s: need 0 <= rank (%d) < nranks, 0 <= max_tokens (%d) <= %d and an all-gather callback", what,
                      rank, max_tokens, TYB_MAX_SEQ);
        return 1;
    }
    if (g_sh.active) {
        tyb_set_error("%s: already set up (attn_shard_close first)", what);
        return 1;
    }
    memset(&g_sh, 0, sizeof g_sh);
    g_sh.rank = rank;
    g_sh.nranks = nranks;
    g_sh.max_tokens = max_tokens;
    unsigned char mine[2 * TYB_IPC_HANDLE_BYTES];
    memset(mine, 0, sizeof mine);
    if (!tyb_cuda_ok(tyb_gather_init(rank, nranks), what) || !tyb_cuda_ok(tyb_gather_handle(mine), what)) {
        tyb_gather_close();
        return 1;
    }
    g_sh.active = 1; /* shard_release undoes everything from here on */
    const size_t slot_elems = (size_t)max_tokens * 16 * KV_HEAD_DIM;
    if (max_tokens > 0) {
        const size_t bytes = TYB_PX_HEADER_BYTES + 2 * slot_elems * 2;
        if (!tyb_dev_alloc(&g_sh.px, bytes, "attn_shard_init: prefill exchange") ||
            !tyb_cuda_ok(cudaMemset(g_sh.px, 0, TYB_PX_HEADER_BYTES), what)) {
            shard_release();
            return 1;
        }
        cudaIpcMemHandle_t h;
        if (!tyb_cuda_ok(cudaIpcGetMemHandle(&h, g_sh.px), what)) {
            shard_release();
            return 1;
        }
        memcpy(mine + TYB_IPC_HANDLE_BYTES, &h, sizeof h);
    }
    unsigned char *all = (unsigned char *)malloc((size_t)nranks * sizeof mine);
    unsigned char *dec = (unsigned char *)malloc((size_t)nranks * TYB_IPC_HANDLE_BYTES);
    if (!all || !dec) {
        free(all);
        free(dec);
        tyb_set_error("%s: out of host memory", what);
        shard_release();
        return 1;
    }
    int ok = allgather(mine, all, sizeof mine, user) == 0;
    if (!ok) tyb_set_error("%s: the all-gather callback failed", what);
    for (int p = 0; ok && p < nranks; p++)
        memcpy(dec + (size_t)p * TYB_IPC_HANDLE_BYTES, all + (size_t)p * sizeof mine, TYB_IPC_HANDLE_BYTES);
    ok = ok && tyb_cuda_ok(tyb_gather_connect(dec), what);
    if (ok && max_tokens > 0) {
        tyb_prefill_x table;
        memset(&table, 0, sizeof table);
        table.rank = rank;
        table.world = nranks;
        table.slot_elems = (long long)slot_elems;
        for (int p = 0; ok && p < nranks; p++) {
            if (p == rank) {
                g_sh.peer_px[p] = g_sh.px;
            } else {
                cudaIpcMemHandle_t h;
                memcpy(&h, all + (size_t)p * sizeof mine + TYB_IPC_HANDLE_BYTES, sizeof h);
                ok = tyb_cuda_ok(cudaIpcOpenMemHandle(&g_sh.peer_px[p], h, cudaIpcMemLazyEnablePeerAccess), what);
                if (!ok) g_sh.peer_px[p] = NULL;
            }
            table.base[p] = g_sh.peer_px[p];
        }
        ok = ok && tyb_dev_alloc((void **)&g_sh.px_dev, sizeof table, "attn_shard_init: exchange table") &&
             tyb_cuda_ok(cudaMemcpy(g_sh.px_dev, &table, sizeof table, cudaMemcpyHostToDevice), what) &&
             tyb_cuda_ok(tyb_prefill_x_maps(table.base, nranks, max_tokens, g_sh.px_maps), what);
    }
    free(all);
    free(dec);
    if (!ok) {
        shard_release();
        return 1;
    }
    return 0;
}

void attn_shard_close(void)
{
    if (g_sh.active) shard_release();
}

int attn_shard_heads(int *kv_head0, int *kv_heads)
{
    if (!g_sh.active) {
        tyb_set_error("attn_shard_heads: no sharding set up (attn_shard_init)");
        return 1;
    }
    const int n = KV_NUM_KV_HEADS / g_sh.nranks;
    if (kv_head0) *kv_head0 = g_sh.rank * n;
    if (kv_heads) *kv_heads = n;
    return 0;
}

int attention_decode_append_gqa_sharded(const float *q, const float *k_new, const float *v_new, KVCache *cache,
                                        float *output, int layer_idx, float scale)
{
    int h0, n;
    if (attn_shard_heads(&h0, &n)) return 1;
    return attention_decode_append_gqa_gathered(q, k_new, v_new, cache, output, layer_idx, scale, h0, n);
}

int attention_prefill_fused_gqa_sharded(const void *q_raw, const void *k_raw, const void *v_raw, int in_dtype,
                                        const float *q_norm, const float *k_norm, const float *token_cos,
                                        const float *token_sin, KVCache *cache, int layer_idx, int seq_len,
                                        float scale, float eps, void **output)
{
    const char *what = "attention_prefill_fused_gqa_sharded";
    int h0, n;
    if (attn_shard_heads(&h0, &n)) return 1;
    if (!output) {
        tyb_set_error("%s: NULL output", what);
        return 1;
    }
    if (seq_len < 0 || seq_len > g_sh.max_tokens) {
        tyb_set_error("%s: seq_len %d exceeds the max_tokens (%d) of attn_shard_init", what, seq_len, g_sh.max_tokens);
        return 1;
    }
    const unsigned int epoch = g_sh.px_epoch + 1u;
    const size_t slot_bytes = (size_t)g_sh.max_tokens * 16 * KV_HEAD_DIM * 2;
    void *slot = (char *)g_sh.px + TYB_PX_HEADER_BYTES + (size_t)(epoch & 1u) * slot_bytes;
    if (seq_len == 0) {
        *output = slot;
        return 0;
    }
    if (tyb_prefill_sharded(q_raw, k_raw, v_raw, in_dtype, q_norm, k_norm, token_cos, token_sin, cache, layer_idx,
                            slot, seq_len, scale, eps, h0, n, g_sh.px_dev, g_sh.px_maps, epoch, what))
        return 1;
    g_sh.px_epoch = epoch;
    *output = slot;
    return 0;
}
