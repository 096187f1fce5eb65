/*
 * attn_oracle.h -- TEST INFRASTRUCTURE ONLY (never linked into the product).
 *
 * CPU restatement of typhoon-ocr-server's GQA attention hot path, used as the
 * checker for the CUDA kernels.  Every function cites the reference lines it
 * restates (paths relative to the reference project root).  Only tests/, the
 * smoke check in __graft_entry__.py and bench.py's CPU-baseline leg load it.
 *
 * Fixed model constants (kernel/attention.c:43-46, kernel/kv_cache.h:7-9):
 * 16 query heads, 8 KV heads, head_dim 128, GQA group 2.
 *
 * Layouts:
 *   token-major  q/out [S][16][128], k/v [S][8][128]          (kernel/attention.c:27-30)
 *   head-first   cache_k/cache_v [8][max_seq][128] for ONE layer (kernel/kv_cache.h:11-26)
 */
#ifndef ATTN_ORACLE_H
#define ATTN_ORACLE_H

#ifdef __cplusplus
extern "C" {
#endif

/* Causal GQA prefill over token-major q/k/v (kernel/attention.c:252-381). */
void oracle_attention_prefill(const float *q, const float *k, const float *v, float *out,
                              int Sq, int Sk, float scale);

/* Chunked prefill: q token-major, K/V from one layer's head-first cache
 * (kernel/attention.c:413-543). */
void oracle_attention_chunked_prefill(const float *q, const float *cache_k, const float *cache_v,
                                      int max_seq, float *out, int chunk_len, int pos_offset,
                                      float scale);

/* Single-token decode over one layer's head-first cache (kernel/attention.c:158-204). */
void oracle_attention_decode(const float *q, const float *cache_k, const float *cache_v,
                             int max_seq, float *out, int kv_len, float scale);

/* Row-wise RMSNorm (kernel/ops.c:22-62, :99-112); out may alias x. */
void oracle_rmsnorm_rows(float *out, const float *x, const float *weight, int rows, int dim,
                         float eps);

/* Per-token cos/sin [S][64] from 3-D position ids [3][S] (kernel/ops.c:139-155, :195-224). */
void oracle_mrope_cos_sin_3d(float *cos_out, float *sin_out, const int *pos_ids, int seq_len,
                             float theta);

/* Sequential-position table [max_seq][64] (kernel/ops.c:157-181). */
void oracle_mrope_table(float *cos_tab, float *sin_tab, int max_seq, float theta);

/* rotate_half rotary embedding of `heads` rows of 128 with one cos/sin row
 * (kernel/ops.c:236-288, :297-343), in place. */
void oracle_rope_rows(float *x, int heads, const float *cos_row, const float *sin_row);

/* The whole pre-attention chain of kernel/decoder.c:73-93 for a prefill of S
 * tokens with per-token cos/sin: per-head RMSNorm of q and k, then M-RoPE, in place. */
void oracle_qk_norm_rope(float *q, float *k, const float *q_norm, const float *k_norm,
                         const float *token_cos, const float *token_sin, int seq_len, float eps);

#ifdef __cplusplus
}
#endif
#endif
