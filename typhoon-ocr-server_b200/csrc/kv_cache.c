/*
 * kv_cache.c -- the static KV cache of kernel/kv_cache.c (typhoon-ocr-server), resident
 * in HBM.
 *
 * The reference mallocs 28 x 8 x 2 separate float[max_seq][128] arrays
 * (kernel/kv_cache.c:15-34).  Here K and V are each ONE device slab
 * [layer][kv_head][max_seq][128] (fp32 or bf16), and the KVHead pointers point into it,
 * so a (layer, head) row block is contiguous exactly as in the reference and a decode
 * split is one contiguous byte range for a bulk copy.  Row writes from host memory go
 * through a device staging buffer and one scatter kernel (kv_write.cu).
 */
#include <cuda_runtime_api.h>
#include <stdlib.h>
#include <string.h>

#include "attn_ext.h"
#include "host_internal.h"

tyb_cache *tyb_cache_from(const KVCache *c)
{
    if (!c) {
        tyb_set_error("KVCache is NULL");
        return NULL;
    }
    tyb_cache *t = (tyb_cache *)c;
    if (t->magic != TYB_CACHE_MAGIC) {
        tyb_set_error("KVCache was not allocated by kv_cache_alloc of this library");
        return NULL;
    }
    return t;
}

static void cache_release(tyb_cache *t)
{
    if (!t) return;
    cudaFree(t->k_slab);
    cudaFree(t->v_slab);
    cudaFree(t->d_out);
    cudaFree(t->d_kv_stage);
    cudaFree(t->d_partials);
    cudaFree(t->d_counters);
    if (t->h_rows) cudaFreeHost(t->h_rows);
    for (int l = 0; l < KV_NUM_LAYERS; l++)
        if (t->row_ev[l]) cudaEventDestroy((cudaEvent_t)t->row_ev[l]);
    t->magic = 0;
    free(t);
}

KVCache *kv_cache_alloc_ex(int max_seq_len, int kv_dtype)
{
    if (max_seq_len <= 0 || max_seq_len > TYB_MAX_SEQ) {
        tyb_set_error("kv_cache_alloc: max_seq_len must be in [1, %d] (got %d)", TYB_MAX_SEQ, max_seq_len);
        return NULL;
    }
    if (kv_dtype != ATTN_KV_F32 && kv_dtype != ATTN_KV_BF16) {
        tyb_set_error("kv_cache_alloc_ex: unknown kv_dtype %d", kv_dtype);
        return NULL;
    }
    tyb_cache *t = (tyb_cache *)calloc(1, sizeof(tyb_cache));
    if (!t) {
        tyb_set_error("kv_cache_alloc: out of host memory");
        return NULL;
    }
    t->magic = TYB_CACHE_MAGIC;
    t->dtype = kv_dtype == ATTN_KV_BF16 ? TYB_BF16 : TYB_F32;
    t->elem_bytes = kv_dtype == ATTN_KV_BF16 ? 2 : 4;
    t->pub.max_seq_len = max_seq_len;
    t->pub.seq_len = 0;
    t->pub.rope_offset = 0;
    for (int l = 0; l < KV_NUM_LAYERS; l++) t->pending[l] = -1;
    cudaGetDevice(&t->device);
    /* Kernels on this device may flag the status mirror from now on; without one (setup
     * failed) the blocking calls read the status word back each time instead. */
    if (tyb_status_mirror_setup() != 0) cudaGetLastError();

    const size_t slab = (size_t)KV_NUM_LAYERS * KV_NUM_KV_HEADS * max_seq_len * KV_HEAD_DIM * t->elem_bytes;
    /* Upper bound on splits for any kv_len <= max_seq_len: chunks are >= 16 rows. */
    const int nsplit = (max_seq_len + 15) / 16 + 1;
    const size_t part = tyb_decode_partial_floats(1, nsplit) * sizeof(float);

    /* Any failure frees what was allocated and returns NULL (kernel/kv_cache.c:17-30). */
    int ok = tyb_dev_alloc(&t->k_slab, slab, "kv_cache_alloc: K slab") &&
             tyb_dev_alloc(&t->v_slab, slab, "kv_cache_alloc: V slab") &&
             tyb_dev_alloc((void **)&t->d_out, TYB_Q_FLOATS * sizeof(float), "kv_cache_alloc: out") &&
             /* at least 16 KB: a deferred row with its query (TYB_SLOT_FLOATS) is staged here too */
             tyb_dev_alloc((void **)&t->d_kv_stage,
                           2 * (size_t)(max_seq_len < 2 ? 2 : max_seq_len) * TYB_ROW_FLOATS * sizeof(float),
                           "kv_cache_alloc: staging") &&
             tyb_dev_alloc((void **)&t->d_partials, part, "kv_cache_alloc: decode workspace") &&
             tyb_dev_alloc((void **)&t->d_counters, TYB_DEC_WIDE_COUNTER_WORDS * sizeof(unsigned int),
                           "kv_cache_alloc: counters") &&
             tyb_cuda_ok(cudaMemset(t->d_counters, 0, TYB_DEC_WIDE_COUNTER_WORDS * sizeof(unsigned int)),
                         "kv_cache_alloc: counters memset");
    if (!ok) {
        cache_release(t);
        return NULL;
    }
    for (int l = 0; l < KV_NUM_LAYERS; l++)
        for (int h = 0; h < KV_NUM_KV_HEADS; h++) {
            t->pub.layers[l].heads[h].k = (float *)tyb_slab_head(t, t->k_slab, l, h);
            t->pub.layers[l].heads[h].v = (float *)tyb_slab_head(t, t->v_slab, l, h);
        }
    return &t->pub;
}

KVCache *kv_cache_alloc(int max_seq_len) { return kv_cache_alloc_ex(max_seq_len, ATTN_KV_F32); }

int kv_cache_dtype(const KVCache *c)
{
    tyb_cache *t = tyb_cache_from(c);
    if (!t) return -1;
    return t->dtype == TYB_BF16 ? ATTN_KV_BF16 : ATTN_KV_F32;
}

void kv_cache_free(KVCache *c)
{
    if (!c) return;
    tyb_cache *t = tyb_cache_from(c);
    if (!t) return;
    cudaStreamSynchronize((cudaStream_t)tyb_stream());
    cache_release(t);
}

void kv_cache_clear(KVCache *c)
{
    if (!c) return;
    tyb_cache *t = tyb_cache_from(c);
    for (int l = 0; t && l < KV_NUM_LAYERS; l++) tyb_flush_pending(t, l, "kv_cache_clear");
    c->seq_len = 0; /* kernel/kv_cache.c:48-51 */
    c->rope_offset = 0;
}

/* The deferred-append staging (page-locked, mapped) and its per-layer events, on first use. */
int tyb_slots_ready(tyb_cache *t, const char *what)
{
    if (t->h_rows) return 1;
    void *p = NULL;
    if (!tyb_host_alloc(&p, TYB_PINNED_FLOATS * sizeof(float), cudaHostAllocMapped | cudaHostAllocPortable, what))
        return 0;
    memset(p, 0, TYB_PINNED_FLOATS * sizeof(float));
    void *d = NULL;
    if (!tyb_cuda_ok(cudaHostGetDevicePointer(&d, p, 0), what)) {
        cudaFreeHost(p);
        return 0;
    }
    for (int l = 0; l < KV_NUM_LAYERS; l++) {
        cudaEvent_t ev;
        if (!tyb_cuda_ok(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), what)) {
            for (int j = 0; j < l; j++) {
                cudaEventDestroy((cudaEvent_t)t->row_ev[j]);
                t->row_ev[j] = NULL;
            }
            cudaFreeHost(p);
            return 0;
        }
        t->row_ev[l] = ev;
    }
    t->h_rows = (float *)p;
    t->h_rows_dev = (float *)d;
    const size_t out_at = (size_t)KV_NUM_LAYERS * TYB_SLOT_FLOATS;
    t->h_out = t->h_rows + out_at;
    t->h_out_dev = t->h_rows_dev + out_at;
    return 1;
}

int tyb_slot_consumed(tyb_cache *t, int layer, void *stream, const char *what)
{
    if (!tyb_cuda_ok(cudaEventRecord((cudaEvent_t)t->row_ev[layer], (cudaStream_t)stream), what)) return 0;
    t->slot_read[layer] = 1;
    return 1;
}

int tyb_slot_wait(tyb_cache *t, int layer, const char *what)
{
    if (!t->slot_read[layer]) return 1;
    if (!tyb_cuda_ok(cudaEventSynchronize((cudaEvent_t)t->row_ev[layer]), what)) return 0;
    t->slot_read[layer] = 0;
    return 1;
}

int tyb_flush_pending(tyb_cache *t, int layer, const char *what)
{
    const int pos = t->pending[layer];
    if (pos < 0) return 1;
    t->pending[layer] = -1;
    void *st = tyb_stream();
    const float *ks = t->h_rows_dev + (size_t)layer * TYB_SLOT_FLOATS; /* read over the bus */
    void *kl = tyb_slab_head(t, t->k_slab, layer, 0), *vl = tyb_slab_head(t, t->v_slab, layer, 0);
    if (!tyb_cuda_ok(tyb_kv_scatter_launch(ks, ks + TYB_ROW_FLOATS, kl, vl, t->pub.max_seq_len, pos, 1, t->dtype, st),
                     what))
        return 0;
    tyb_note_write(&t->pub, layer, pos, st);
    return tyb_slot_consumed(t, layer, st, what);
}

/* Rows [pos, pos+S) of `layer` from token-major k_new/v_new [S][8][128] fp32. */
static void append_rows(KVCache *c, int layer, const float *k_new, const float *v_new, int S,
                        const char *what)
{
    tyb_cache *t = tyb_cache_from(c);
    if (!t) return;
    if (layer < 0 || layer >= KV_NUM_LAYERS) {
        tyb_set_error("%s: layer %d out of range [0, %d)", what, layer, KV_NUM_LAYERS);
        return;
    }
    const int pos = c->seq_len;
    if (S < 0 || pos < 0 || pos + S > c->max_seq_len) {
        tyb_set_error("%s: rows [%d, %d) exceed max_seq_len %d", what, pos, pos + S, c->max_seq_len);
        return;
    }
    if (S == 0) return;
    if (!k_new || !v_new) {
        tyb_set_error("%s: NULL k_new/v_new", what);
        return;
    }
    const int kd = tyb_is_device_ptr(k_new), vd = tyb_is_device_ptr(v_new);
    if (kd < 0 || vd < 0) return;
    /* An earlier deferred row of this layer lands first (writes keep their order). */
    if (!tyb_flush_pending(t, layer, what)) return;
    if (S == 1 && !kd && !vd) {
        /* One row from host memory, as kernel/decoder.c:96-100 appends each decode step: copied
         * now into the layer's page-locked slot (the caller may reuse its buffers on return, as
         * after the reference's memcpy), written to the cache by the next launch on this layer --
         * attention_decode_gqa over seq_len + 1 rows appends and attends in one kernel. */
        if (tyb_slots_ready(t, what)) {
            if (!tyb_slot_wait(t, layer, what)) return; /* slot free */
            float *slot = tyb_row_slot(t, layer);
            memcpy(slot, k_new, TYB_ROW_FLOATS * sizeof(float));
            memcpy(slot + TYB_ROW_FLOATS, v_new, TYB_ROW_FLOATS * sizeof(float));
            t->pending[layer] = pos;
            return;
        }
        tyb_set_error(""); /* no page-locked slot: the row goes the direct way below */
    }
    void *st = tyb_stream();
    const size_t bytes = (size_t)S * TYB_ROW_FLOATS * sizeof(float);
    const float *ks = k_new, *vs = v_new;
    if (!kd) {
        if (!tyb_cuda_ok(cudaMemcpyAsync(t->d_kv_stage, k_new, bytes, cudaMemcpyHostToDevice, (cudaStream_t)st), what))
            return;
        ks = t->d_kv_stage;
    }
    if (!vd) {
        float *dst = t->d_kv_stage + (size_t)c->max_seq_len * TYB_ROW_FLOATS;
        if (!tyb_cuda_ok(cudaMemcpyAsync(dst, v_new, bytes, cudaMemcpyHostToDevice, (cudaStream_t)st), what))
            return;
        vs = dst;
    }
    void *kl = tyb_slab_head(t, t->k_slab, layer, 0), *vl = tyb_slab_head(t, t->v_slab, layer, 0);
    if (!tyb_cuda_ok(tyb_kv_scatter_launch(ks, vs, kl, vl, c->max_seq_len, pos, S, t->dtype, st), what)) return;
    tyb_note_write(c, layer, pos, st);
    /* Host sources: block until the rows are read, as the reference's memcpy does. */
    if (!kd || !vd) tyb_finish(st, what);
}

void kv_cache_append(KVCache *c, int layer, const float *k_new, const float *v_new)
{
    append_rows(c, layer, k_new, v_new, 1, "kv_cache_append"); /* kernel/kv_cache.c:53-65 */
}

void kv_cache_append_prefill(KVCache *c, int layer, const float *k_new, const float *v_new,
                             int seq_len)
{
    append_rows(c, layer, k_new, v_new, seq_len, "kv_cache_append_prefill"); /* :95-104 */
}

void kv_cache_advance(KVCache *c, int n)
{
    if (!c) return;
    c->seq_len += n; /* kernel/kv_cache.c:106-110 */
    if (c->rope_offset > 0) c->rope_offset += n;
}

/* The rows behind these pointers include a deferred appended row once it is written: it is
 * queued here, before the pointer is handed out. */
const float *kv_cache_k(const KVCache *c, int layer, int head)
{
    tyb_cache *t = tyb_cache_from(c);
    if (t && layer >= 0 && layer < KV_NUM_LAYERS) tyb_flush_pending(t, layer, "kv_cache_k");
    return c->layers[layer].heads[head].k; /* kernel/kv_cache.c:112-115 */
}

const float *kv_cache_v(const KVCache *c, int layer, int head)
{
    tyb_cache *t = tyb_cache_from(c);
    if (t && layer >= 0 && layer < KV_NUM_LAYERS) tyb_flush_pending(t, layer, "kv_cache_v");
    return c->layers[layer].heads[head].v; /* kernel/kv_cache.c:117-120 */
}
