/*
 * scratch.c -- the decoder scratch of kernel/scratch.c (typhoon-ocr-server).
 *
 * Same buffers and aliases as the reference (kernel/scratch.c:22-86).  The token-major
 * activations are written by host code in kernel/decoder.c, so they are page-locked
 * host memory (cudaHostAlloc): transfers to the GPU then run at full link speed and
 * without an extra bounce.  The head-major slots q_hm/k_hm/v_hm/o_hm are device memory
 * and serve attention_prefill_gqa as its staging area.
 */
#include <cuda_runtime_api.h>
#include <stdlib.h>

#include "host_internal.h"
#include "scratch.h"

#define GATE_UP_DIM_S (2 * FFN_DIM)

static void *host_buf(size_t floats, int *ok)
{
    void *p = NULL;
    if (*ok && !tyb_host_alloc(&p, floats * sizeof(float), cudaHostAllocPortable,
                               "decoder_scratch_alloc: pinned host buffer"))
        *ok = 0;
    return p;
}

static float *dev_buf(size_t floats, int *ok)
{
    void *p = NULL;
    if (*ok && tyb_dev_alloc(&p, floats * sizeof(float), "decoder_scratch_alloc: device buffer"))
        tyb_registry_add(p, floats * sizeof(float));
    else
        *ok = 0;
    return (float *)p;
}

DecoderScratch *decoder_scratch_alloc(int max_seq_len)
{
    if (max_seq_len <= 0) {
        tyb_set_error("decoder_scratch_alloc: max_seq_len must be positive (got %d)", max_seq_len);
        return NULL;
    }
    DecoderScratch *s = (DecoderScratch *)calloc(1, sizeof(DecoderScratch));
    if (!s) {
        tyb_set_error("decoder_scratch_alloc: out of host memory");
        return NULL;
    }
    const size_t n = (size_t)max_seq_len;
    int ok = 1;
    s->residual = host_buf(n * HIDDEN_DIM, &ok);
    s->q = host_buf(n * HIDDEN_DIM, &ok);
    s->k = host_buf(n * KV_DIM_SIZE, &ok);
    s->v = host_buf(n * KV_DIM_SIZE, &ok);
    s->attn = host_buf(n * HIDDEN_DIM, &ok);
    s->gate = host_buf(n * FFN_DIM, &ok);
    s->up = host_buf(n * FFN_DIM, &ok);
    s->mlp = s->gate;       /* alias (kernel/scratch.c:41) */
    s->qkv_fused = s->gate; /* alias (kernel/scratch.c:53) */
    s->gate_up_fused = host_buf(n * GATE_UP_DIM_S, &ok);
    s->q_hm = dev_buf((size_t)NUM_Q_HEADS_S * n * HEAD_DIM_QK, &ok);
    s->k_hm = dev_buf((size_t)NUM_KV_HEADS_S * n * HEAD_DIM_QK, &ok);
    s->v_hm = dev_buf((size_t)NUM_KV_HEADS_S * n * HEAD_DIM_QK, &ok);
    s->o_hm = dev_buf((size_t)NUM_Q_HEADS_S * n * HEAD_DIM_QK, &ok);
    if (!ok) {
        decoder_scratch_free(s); /* frees what was allocated (kernel/scratch.c:58-64) */
        return NULL;
    }
    return s;
}

void decoder_scratch_free(DecoderScratch *s)
{
    if (!s) return;
    cudaStreamSynchronize((cudaStream_t)tyb_stream());
    cudaFreeHost(s->residual);
    cudaFreeHost(s->q);
    cudaFreeHost(s->k);
    cudaFreeHost(s->v);
    cudaFreeHost(s->attn);
    cudaFreeHost(s->gate);
    cudaFreeHost(s->up);
    cudaFreeHost(s->gate_up_fused);
    /* mlp and qkv_fused alias gate: not freed separately (kernel/scratch.c:83-84). */
    float *dev[4] = {s->q_hm, s->k_hm, s->v_hm, s->o_hm};
    for (int i = 0; i < 4; i++)
        if (dev[i]) {
            tyb_registry_remove(dev[i]);
            cudaFree(dev[i]);
        }
    free(s);
}
