/*
 * attn_ext.h -- additions to the reference interface (none of these exist in
 * typhoon-ocr-server; the reference's attention/append functions return void and
 * have no error channel, kernel/attention.h:11,26,39).
 */
#pragma once
#include <stddef.h>

#include "kv_cache.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Element type of KV-cache rows. */
#define ATTN_KV_F32  0
#define ATTN_KV_BF16 1

/* Like kv_cache_alloc, with the row element type chosen.  ATTN_KV_BF16 halves the
 * bytes decode streams; its parity bar against the FP32 reference is the BF16 one. */
KVCache *kv_cache_alloc_ex(int max_seq_len, int kv_dtype);
/* ATTN_KV_F32 or ATTN_KV_BF16; -1 for a pointer this library did not allocate. */
int      kv_cache_dtype(const KVCache *c);

/* Last error of the calling thread ("" when none), and clearing it.  Set by every
 * entry point of this library on bad arguments, CUDA errors and device status bits
 * (a kernel wait that ran out of time, an index check that failed). */
const char *attn_last_error(void);
void        attn_clear_error(void);

/* Stream (a cudaStream_t) for subsequent device work of this thread's calls; NULL
 * selects the legacy default stream (the initial setting). */
void attn_set_stream(void *stream);
/* Wait for all queued work on the library stream, then check the device status word.
 * 0 on success, else nonzero with attn_last_error() set. */
int  attn_sync(void);

/* Limit, in nanoseconds, of every bounded wait in this library's kernels on the current device
 * (a tile copy that never lands, a peer rank that never raises its flag); 2 s until set.  A wait
 * that runs out ends its kernel early with a device status bit, which the next blocking call or
 * attn_sync() reports through attn_last_error() ("wait timed out"); the CUDA context stays
 * usable.  Applies to kernels launched afterwards.  ns >= 1000.  0 on success. */
int attn_set_wait_limit_ns(unsigned long long ns);

/* Sizes the current device's workspace now, so that later calls within these sizes allocate
 * nothing: the staging of host buffers and the K/V operand splits of attention_prefill_gqa
 * without scratch slots and of attention_chunked_prefill_gqa (max_tokens query tokens), and the
 * descriptors, staging and split records of attention_decode_gqa_batched (max_batch sequences of
 * at most max_kv_len rows).  Without it the first call that needs more grows the workspace
 * (after waiting for the device).  The workspace is per device; calls from several host threads
 * on one device share it and must not overlap.  0 on success. */
int attn_workspace_reserve(int max_tokens, int max_batch, int max_kv_len);

/* Decode for `batch` independent sequences in one launch (request-level batching;
 * ragged kv lengths).  q, output: [batch][16][128] fp32 (host or device);
 * caches[b]: the cache of sequence b (all with the same element type);
 * kv_lens[b]: rows attended for sequence b.  0 on success. */
int attention_decode_gqa_batched(const float *q, const KVCache *const *caches,
                                 const int *kv_lens, float *output, int batch,
                                 int layer_idx, float scale);

/* Element types of the fused prefill's activations. */
#define ATTN_DT_F32  0
#define ATTN_DT_BF16 1

/* One layer of the multimodal prefill chain of kernel/decoder.c:73-117 in two launches, on
 * the tensor cores: RMSNorm of q and k with q_norm/k_norm (eps), rotate_half M-RoPE with the
 * per-token tables token_cos/token_sin [seq_len][64] (from decoder_build_rope_3d), K/V
 * appended to the cache at rows cache->seq_len.., then causal attention of the seq_len new
 * queries over cache rows [0, cache->seq_len + seq_len) -- query i at position
 * cache->seq_len + i (a fresh cache gives the plain prefill; a filled one, chunked prefill).
 * q_raw [seq_len][16][128], k_raw/v_raw [seq_len][8][128] in `in_dtype`; output
 * [seq_len][16][128] in `out_dtype`; q_norm/k_norm [128] fp32.  All DEVICE memory; the cache
 * must be ATTN_KV_BF16.  BF16 operands, FP32 accumulation (tolerance of the BF16 path).
 * seq_len is not advanced.  0 on success. */
int attention_prefill_fused_gqa(const void *q_raw, const void *k_raw, const void *v_raw, int in_dtype,
                                const float *q_norm, const float *k_norm, const float *token_cos,
                                const float *token_sin, KVCache *cache, int layer_idx, void *output,
                                int out_dtype, int seq_len, float scale, float eps);

/* One decode step of one layer in one launch: kv_cache_append(cache, layer_idx, k_new, v_new)
 * followed by attention_decode_gqa(q, cache, output, layer_idx, cache->seq_len + 1, scale)
 * (kernel/kv_cache.c:53-65, kernel/attention.c:194-204; the pair kernel/decoder.c:97,104
 * calls).  The new row is written to the cache and used directly, so the kernel can
 * start streaming the older rows before the previous kernel in the stream finishes.
 * seq_len is not advanced (kv_cache_advance does that, as in the reference).
 * q, output [16][128]; k_new, v_new [8][128]; fp32, host or device.  0 on success.
 * Rows of the cache are assumed to be written only through this library's calls (or by
 * work that has completed before the call is made). */
int attention_decode_append_gqa(const float *q, const float *k_new, const float *v_new,
                                KVCache *cache, float *output, int layer_idx, float scale);

/* One decode step of one layer with the whole of kernel/decoder.c:73-105 on the GPU: RMSNorm of
 * the raw query heads with q_norm and of the raw key heads with k_norm (eps), rotate_half M-RoPE
 * of both with the token's token_cos / token_sin [64] (one row of the per-token tables; for text
 * decode all three sections share the position rope_offset or seq_len, kernel/decoder.c:80-83),
 * the normed, rotated key row and v_new appended at row cache->seq_len, then the attention of
 * the query over rows [0, seq_len + 1).  The normalisation and rotation run inside the decode
 * kernel as it loads q and the new row, so the host no longer runs rmsnorm_f32 /
 * mrope_apply_token per step.  q_raw [16][128], k_raw and v_new [8][128], q_norm / k_norm [128],
 * token_cos / token_sin [64], output [16][128]: fp32, all DEVICE memory (queued on the library
 * stream; attn_sync waits).  The cache must be ATTN_KV_BF16.  seq_len is not advanced.  0 on
 * success. */
int attention_decode_append_fused_gqa(const float *q_raw, const float *k_raw, const float *v_new,
                                      const float *q_norm, const float *k_norm, const float *token_cos,
                                      const float *token_sin, KVCache *cache, float *output, int layer_idx,
                                      float scale, float eps);

/* ---- KV-head sharding (one long sequence over N GPUs) ---------------------------------
 * The GQA heads are independent: KV head h and query heads 2h, 2h+1 need no other head.  A
 * long sequence is split over N GPUs by KV head (8/N each); every GPU holds its heads'
 * rows of the cache and computes its query heads' outputs as one contiguous shard, the
 * shards are all-gathered (ncclAllGather in rank order, by the caller) into head-major
 * [16][S][128], and attn_heads_to_tokens turns that into the token-major layout decoder.c
 * uses.  The reference has no multi-GPU path; these extend attention_prefill_fused_gqa and
 * attention_decode_append_gqa.  kv_head0, kv_heads:
 * the KV heads [kv_head0, kv_head0 + kv_heads) computed here, 1 <= kv_heads <= 8.
 *
 * attention_prefill_fused_gqa for the given KV heads only (their K/V rows appended, their
 * query heads' attention); inputs as there (the full q_raw/k_raw/v_raw; the other heads are
 * not read); output the shard [2 kv_heads][seq_len][128] in out_dtype.  0 on success. */
int attention_prefill_fused_gqa_heads(const void *q_raw, const void *k_raw, const void *v_raw, int in_dtype,
                                      const float *q_norm, const float *k_norm, const float *token_cos,
                                      const float *token_sin, KVCache *cache, int layer_idx, void *output,
                                      int out_dtype, int seq_len, float scale, float eps, int kv_head0,
                                      int kv_heads);

/* attention_decode_append_gqa for the given KV heads only: output the shard [2 kv_heads][128]
 * (query heads 2 kv_head0 ..), host or device.  0 on success. */
int attention_decode_append_gqa_heads(const float *q, const float *k_new, const float *v_new,
                                      KVCache *cache, float *output, int layer_idx, float scale,
                                      int kv_head0, int kv_heads);

/* Decode output gather over NVLink, without a collective library: attention_decode_append_gqa_heads
 * whose output is the whole [16][128] on every rank, in one launch.  The CTA that finishes a head
 * pair stores it into every rank's exchange buffer (peer stores into memory mapped by CUDA IPC),
 * each value as a 64-bit word carrying the call's number; the rank's last such CTA reads the
 * 16 x 128 words of its own buffer, each until it carries the call's number (bounded;
 * attn_last_error on timeout), and writes the values to `output`.  One rank per
 * GPU on one node, up to 8 ranks; every rank calls with the same layers in the same order, and
 * the ranks' KV-head ranges together cover the 8 heads.
 *   attn_gather_init(rank, world)   allocates this rank's exchange buffer on the current device
 *   attn_gather_handle(h)           writes its 64-byte CUDA IPC handle to h
 *   attn_gather_connect(handles)    handles: world x 64 bytes in rank order (exchanged by the
 *                                   caller, e.g. with torch.distributed); maps the peers' buffers
 *   attn_gather_close()             unmaps and frees (after all calls have completed)
 * attention_decode_append_gqa_gathered: as attention_decode_append_gqa_heads for the KV heads
 * [kv_head0, kv_head0 + kv_heads) of this rank (BF16 cache), output [16][128] fp32 (host or
 * device).  0 on success. */
int  attn_gather_init(int rank, int world);
int  attn_gather_handle(void *handle_out);
int  attn_gather_connect(const void *handles);
void attn_gather_close(void);
int  attention_decode_append_gqa_gathered(const float *q, const float *k_new, const float *v_new, KVCache *cache,
                                          float *output, int layer_idx, float scale, int kv_head0, int kv_heads);

/* ---- KV-head sharding set up from C (one rank per GPU on one node) ----------------------
 * The pieces above, tied together without a collective library:
 *
 * attn_allgather_fn: an all-gather the caller supplies -- `bytes` bytes from every rank, written
 * to recv in rank order (recv[r * bytes ..] = rank r's send) -- e.g. MPI_Allgather, a TCP store, or
 * torch.distributed.  Called once, by attn_shard_init, for 128 bytes per rank.  0 on success.
 *
 * attn_shard_init(rank, nranks, max_tokens, allgather, user): rank `rank` of `nranks` (1, 2, 4
 * or 8) owns KV heads [8 rank / nranks, 8 (rank + 1) / nranks).  Allocates on the current device
 * the decode output exchange and a prefill output exchange for sequences of up to max_tokens
 * tokens (2 x max_tokens x 4 KB: two BF16 slots), exchanges the CUDA IPC handles through
 * `allgather` and maps every peer's buffers.  Every rank calls it, then makes the same calls in
 * the same order.  0 on success.  attn_shard_close(): after all calls have completed.
 * attn_shard_heads: this rank's KV heads.
 *
 * attention_prefill_fused_gqa_sharded: attention_prefill_fused_gqa_heads for this rank's KV heads
 * (raw inputs as there; BF16 cache), whose tensor-core kernel stores every output tile, token-major
 * BF16, into the exchange buffer of EVERY rank (TMA stores over NVLink from the epilogue that
 * produces it) and returns once all ranks' rows are in place: *output receives this rank's
 * device address of the assembled [seq_len][16][128] BF16 output, valid until the call after
 * next (two slots).  seq_len <= max_tokens.  Calls count on the host: not for CUDA graph
 * capture.  0 on success.
 *
 * attention_decode_append_gqa_sharded: attention_decode_append_gqa_gathered for this rank's KV
 * heads (output [16][128] on every rank).  0 on success. */
typedef int (*attn_allgather_fn)(const void *send, void *recv, size_t bytes, void *user);
int  attn_shard_init(int rank, int nranks, int max_tokens, attn_allgather_fn allgather, void *user);
void attn_shard_close(void);
int  attn_shard_heads(int *kv_head0, int *kv_heads);
int  attention_prefill_fused_gqa_sharded(const void *q_raw, const void *k_raw, const void *v_raw, int in_dtype,
                                         const float *q_norm, const float *k_norm, const float *token_cos,
                                         const float *token_sin, KVCache *cache, int layer_idx, int seq_len,
                                         float scale, float eps, void **output);
int  attention_decode_append_gqa_sharded(const float *q, const float *k_new, const float *v_new, KVCache *cache,
                                         float *output, int layer_idx, float scale);

/* Gathered head-major [16][seq_len][128] -> token-major [seq_len][16][128], in dtype
 * (ATTN_DT_F32 or ATTN_DT_BF16); device memory, queued on the library stream.  0 on success. */
int attn_heads_to_tokens(const void *gathered, void *output, int seq_len, int dtype);

/* No counterpart in the reference.  Decode attention for one sequence and one layer that
 * allocates no memory, for callers that cannot call cudaMalloc: a serving engine whose
 * device memory is all reserved up front by its own caching allocator (an allocation behind
 * its back can fail or fragment that pool), or a program that keeps a fixed, audited
 * device-memory footprint.  Its scratch is a fixed array of about 2 MiB that exists on every
 * GPU that loads this library until the process exits.
 *   q, output       device [16][128] fp32
 *   k_rows, v_rows  device, head-first [8][row_capacity][128] of kv_dtype (ATTN_KV_F32 or
 *                   ATTN_KV_BF16), 16-byte aligned -- e.g. kv_cache_k(cache, layer, 0)
 *   kv_len          rows attended, 1 <= kv_len <= row_capacity; for ATTN_KV_F32 at most 24,576
 *                   rows (256 splits of 96; longer requests are rejected); ATTN_KV_BF16 has no
 *                   such limit (long sequences are streamed in at most 2 x SMs / 8 spans)
 *   stream          cudaStream_t (NULL = legacy default stream); the call only queues work
 * The first call on each device looks up the array's device address (cudaGetSymbolAddress);
 * make that first call before any stream capture.  The address is kept until the process exits,
 * so this entry point must not be used on a device after cudaDeviceReset there (reload the
 * library first).  All calls share the one array and it
 * keeps the last call's contents: calls that overlap on the GPU (other streams, other
 * threads) race, so serialise them, e.g. on one stream.  0 on success, else nonzero with
 * attn_last_error() set. */
int attention_decode_gqa_noalloc(const float *q, const void *k_rows, const void *v_rows,
                                 int row_capacity, int kv_dtype, float *output, int kv_len,
                                 float scale, void *stream);

#ifdef __cplusplus
}
#endif
