/*
 * attention.h -- GQA attention entry points, executed by sm_100a kernels.
 *
 * Drop-in for the reference interface kernel/attention.h:1-47 of typhoon-ocr-server:
 * same names, arguments and meaning.  Fixed model: 16 query heads, 8 KV heads,
 * head_dim 128, query head h reads KV head h/2.
 *
 * Memory: every float pointer may be host memory (pageable or pinned) or device
 * memory; the library detects which.  With any host buffer the call returns only
 * when its outputs are written (the reference's blocking contract).  With device
 * buffers only, work is queued on the library stream (attn_set_stream) and
 * attn_sync() waits for it.  Errors go to attn_last_error() (attn_ext.h), since these
 * functions return void like the reference's.
 */
#pragma once
#include "kv_cache.h"

#ifdef __cplusplus
extern "C" {
#endif

/* kernel/attention.h:11-18 -- one new token.
 * q, output: [NUM_Q_HEADS × HEAD_DIM] fp32.
 * kv_len: rows attended, including the one just appended (typically cache->seq_len + 1). */
void attention_decode_gqa(
    const float  *q,
    const KVCache *cache,
    float         *output,
    int layer_idx,
    int kv_len,
    float scale
);

/* kernel/attention.h:26-33 -- causal prefill over token-major q [Sq][16][128] and
 * k, v [Sk][8][128] (fp32), output [Sq][16][128].  Query i attends keys 0..i (< Sk).
 * q_hm/k_hm/v_hm/o_hm: the reference reserved them for a zero-copy path; here, when
 * they are device buffers of the DecoderScratch sizes, they stage host inputs and the
 * output on the device; otherwise (NULL or host memory) an internal workspace does.  With
 * q/k/v/output all in host memory and Sk >= Sq >= 1024, the rows cross the bus in chunks that
 * overlap the kernels and each other (two copy streams of the calling thread); the call still
 * returns once the output is written. */
void attention_prefill_gqa(
    const float  *q,
    const float  *k,
    const float  *v,
    float         *output,
    int Sq, int Sk, float scale,
    float *q_hm, float *k_hm, float *v_hm, float *o_hm
);

/* kernel/attention.h:39-47 -- q token-major [chunk_len][16][128]; K/V from the cache
 * rows [0, pos_offset + chunk_len) of `layer_idx`; query i sits at pos_offset + i. */
void attention_chunked_prefill_gqa(
    const float  *q,
    const KVCache *cache,
    float         *output,
    int layer_idx,
    int chunk_len,
    int pos_offset,
    float scale
);

#ifdef __cplusplus
}
#endif
