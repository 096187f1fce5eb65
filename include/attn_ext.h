/*
 * attn_ext.h -- additions to the reference interface (none of these exist in
 * typhoon-ocr-server; the reference's attention/append functions return void and
 * have no error channel, kernel/attention.h:11,26,39).
 */
#pragma once
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

/* Decode for `batch` independent sequences in one launch (request-level batching;
 * ragged kv lengths).  q, output: [batch][16][128] fp32 (host or device);
 * caches[b]: the cache of sequence b (all with the same element type);
 * kv_lens[b]: rows attended for sequence b.  0 on success. */
int attention_decode_gqa_batched(const float *q, const KVCache *const *caches,
                                 const int *kv_lens, float *output, int batch,
                                 int layer_idx, float scale);

#ifdef __cplusplus
}
#endif
