/*
 * scratch.h -- pre-allocated decoder scratch: pinned host activations plus a device
 * staging workspace.
 *
 * Drop-in for the reference interface kernel/scratch.h:1-37 of typhoon-ocr-server:
 * same constants, same DecoderScratch field order, same alloc/free signatures.
 * kernel/decoder.c writes q, k, v, attn, gate, up, mlp, qkv_fused, gate_up_fused and
 * residual from host code, so those stay HOST memory -- page-locked here, so copies to
 * and from the GPU run at full PCIe/C2C speed.  The head-major slots q_hm, k_hm, v_hm,
 * o_hm, "reserved for a future zero-copy path" in the reference (kernel/attention.h:25),
 * become DEVICE buffers: attention_prefill_gqa stages q/k/v and its output through them.
 * mlp and qkv_fused alias gate (kernel/scratch.c:41,53) and are not freed separately.
 */
#pragma once
#include <stddef.h>

/* Qwen3-VL 2B decoder dimensions */
#define HIDDEN_DIM  2048
#define KV_DIM_SIZE 1024   /* num_kv_heads(8) × head_dim(128) */
#define FFN_DIM     6144
#define NUM_Q_HEADS_S  16
#define NUM_KV_HEADS_S  8
#define HEAD_DIM_QK   128

typedef struct {
    float *residual;  /* [max_seq × HIDDEN_DIM]  — token-major (pinned host) */
    float *q;         /* [max_seq × HIDDEN_DIM]  — token-major, after linear+norm+rope */
    float *k;         /* [max_seq × KV_DIM_SIZE] — token-major */
    float *v;         /* [max_seq × KV_DIM_SIZE] — token-major */
    float *attn;      /* [max_seq × HIDDEN_DIM]  — token-major attention output */
    float *gate;      /* [max_seq × FFN_DIM]     */
    float *up;        /* [max_seq × FFN_DIM]     */
    float *mlp;       /* aliases gate after SwiGLU */
    /* Device staging buffers (head-major slots of the reference) */
    float *q_hm;      /* [NUM_Q_HEADS  × max_seq × HEAD_DIM] (device) */
    float *k_hm;      /* [NUM_KV_HEADS × max_seq × HEAD_DIM] (device) */
    float *v_hm;      /* [NUM_KV_HEADS × max_seq × HEAD_DIM] (device) */
    float *o_hm;      /* [NUM_Q_HEADS  × max_seq × HEAD_DIM] (device) */
    float *qkv_fused;      /* aliases gate */
    float *gate_up_fused;  /* [max_seq × 12288] */
} DecoderScratch;

#ifdef __cplusplus
extern "C" {
#endif

/* kernel/scratch.h:36 -- NULL on failure after freeing what was allocated. */
DecoderScratch *decoder_scratch_alloc(int max_seq_len);
/* kernel/scratch.h:37 */
void            decoder_scratch_free(DecoderScratch *s);

#ifdef __cplusplus
}
#endif
