/*
 * kv_cache.h -- static KV cache, device-resident on a B200.
 *
 * Drop-in for the reference interface kernel/kv_cache.h:1-38 of typhoon-ocr-server:
 * the constants, the KVHead/KVLayer/KVCache layout and every signature are unchanged,
 * so kernel/decoder.c (which reads and writes cache->seq_len and cache->rope_offset
 * directly, decoder.c:80,92,105,108,115,349) compiles and runs against it as is.
 *
 * What changes is where the rows live: KVHead.k / KVHead.v are DEVICE pointers into one
 * HBM slab per tensor, laid out [layer 28][kv_head 8][max_seq_len][128].  They are typed
 * float* for ABI compatibility; a cache made with kv_cache_alloc_ex(.., ATTN_KV_BF16)
 * holds bf16 rows behind the same pointers.  seq_len / max_seq_len / rope_offset stay
 * host ints at their reference offsets.
 */
#pragma once
#include <stdint.h>

/* Qwen3-VL 2B decoder constants */
#define KV_NUM_LAYERS    28
#define KV_NUM_KV_HEADS   8
#define KV_HEAD_DIM     128

typedef struct {
    float *k;   /* [max_seq × head_dim] — contiguous per head per layer (device) */
    float *v;   /* [max_seq × head_dim] (device) */
} KVHead;

typedef struct {
    KVHead heads[KV_NUM_KV_HEADS];
} KVLayer;

typedef struct {
    KVLayer layers[KV_NUM_LAYERS];
    int     seq_len;
    int     max_seq_len;
    int     rope_offset;  /* decode RoPE position = rope_offset + decode_step */
} KVCache;

#ifdef __cplusplus
extern "C" {
#endif

/* kernel/kv_cache.h:28 -- FP32 device cache; NULL on failure (attn_last_error says why). */
KVCache      *kv_cache_alloc(int max_seq_len);
/* kernel/kv_cache.h:29 */
void          kv_cache_free(KVCache *c);
/* kernel/kv_cache.h:30 -- seq_len = rope_offset = 0 (rows are not cleared, as in the reference). */
void          kv_cache_clear(KVCache *c);
/* kernel/kv_cache.h:31 -- writes row seq_len of every KV head of `layer` from
 * k_new/v_new [8][128] fp32, host or device memory. */
void          kv_cache_append(KVCache *c, int layer,
                              const float *k_new, const float *v_new);
/* kernel/kv_cache.h:32-34 -- writes rows [seq_len, seq_len+seq_len_new) from token-major
 * [seq_len_new][8][128] fp32, host or device memory. */
void          kv_cache_append_prefill(KVCache *c, int layer,
                                      const float *k_new, const float *v_new,
                                      int seq_len);
/* kernel/kv_cache.h:35 -- seq_len += n; rope_offset += n only if already > 0. */
void          kv_cache_advance(KVCache *c, int n);
/* kernel/kv_cache.h:36-37 -- device pointer to the head's first row. */
const float  *kv_cache_k(const KVCache *c, int layer, int head);
const float  *kv_cache_v(const KVCache *c, int layer, int head);

#ifdef __cplusplus
}
#endif
