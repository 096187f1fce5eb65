/*
 * attention.c -- the attention entry points of kernel/attention.h (typhoon-ocr-server),
 * as host C that stages memory and launches the sm_100a kernels.
 *
 *   attention_decode_gqa          kernel/attention.c:194-204  -> decode.cu
 *   attention_prefill_gqa         kernel/attention.c:364-381  -> prefill_tc32.cu (tensor cores,
 *                                                                 FP32-accurate hi/lo splits)
 *   attention_chunked_prefill_gqa kernel/attention.c:527-543  -> prefill_tc32.cu, K/V
 *                                                                 from the device cache
 *   attention_decode_gqa_batched  (new)                       -> decode.cu, many caches
 *   attention_decode_append_gqa   (new) kernel/kv_cache.c:53-65 + attention.c:194-204
 *                                                             -> decode.cu, fused
 *
 * Host buffers are copied to the device on the library stream and results copied back,
 * and then the call waits: the reference's calls block until done.  The single-token decode
 * calls take host inputs as the launch's parameter block instead (inline_inputs) and return
 * once their host output's words are written (host_output, tyb_wait_output).  Device buffers
 * are used in place and the call returns once the work is queued.
 */
#include <cuda_runtime_api.h>
#include <stdlib.h>
#include <string.h>

#include "attention.h"
#include "attn_ext.h"
#include "host_internal.h"

/* flags: TYB_DEC_DEVICE_SMALL when q is device memory (not a mapped page-locked host buffer). */
static int decode_launch(const float *q, float *out, const tyb_seq_kv *seqs_dev, tyb_seq_kv one, int batch,
                         int max_kv, int dtype, float scale, int prefetch_rows, float *partials,
                         unsigned int *counters, int flags, const float *inl, void *st)
{
    return tyb_decode_launch_heads(q, out, seqs_dev, one, batch, max_kv, dtype, scale, partials, counters, NULL, NULL,
                                   prefetch_rows, 0, KV_NUM_KV_HEADS, flags, NULL, inl, st);
}

static int check_layer(int layer, const char *what)
{
    if (layer < 0 || layer >= KV_NUM_LAYERS) {
        tyb_set_error("%s: layer_idx %d out of range [0, %d)", what, layer, KV_NUM_LAYERS);
        return 0;
    }
    return 1;
}

/* Device view of `p`: p itself if it is device memory, else `stage` after an H2D copy
 * of `bytes` (stage == NULL: only report residency).  Returns NULL on error. */
static const float *to_device(const float *p, float *stage, size_t bytes, int *is_dev, void *st,
                              const char *what)
{
    int d = tyb_is_device_ptr(p);
    if (d < 0) return NULL;
    *is_dev = d;
    if (d) return tyb_aligned16(p, what) ? p : NULL;
    if (bytes && !tyb_cuda_ok(cudaMemcpyAsync(stage, p, bytes, cudaMemcpyHostToDevice, (cudaStream_t)st), what))
        return NULL;
    return stage;
}

/* Device view of a small per-call buffer: device memory in place, page-locked host memory
 * through its device mapping (the kernel reads or writes it over the bus: no copy to queue
 * and wait for), pageable host memory through `stage` after an H2D copy of `bytes` (stage
 * == NULL: a result buffer, copied back by the caller).  *kind receives TYB_MEM_*.  NULL on
 * error. */
static float *small_view(const float *p, float *stage, size_t bytes, int *kind, void *st, const char *what)
{
    void *view = NULL;
    const int k = tyb_residency(p, &view);
    *kind = k;
    if (k < 0) return NULL;
    if (k != TYB_MEM_HOST) return tyb_aligned16(view, what) ? (float *)view : NULL;
    if (stage && !tyb_cuda_ok(cudaMemcpyAsync(stage, p, bytes, cudaMemcpyHostToDevice, (cudaStream_t)st), what))
        return NULL;
    return stage;
}

static int decode_append_impl(const float *q, const float *k_new, const float *v_new, KVCache *cache, float *output,
                              int layer_idx, float scale, int kvh0, int nkvh, const void *gather, int pos_at,
                              const char *what);

/* Host inputs of a one-sequence decode call: when q and, for an append, k_new / v_new are all
 * host memory (page-locked or not), they are copied into the layer's page-locked slot
 * [K row][V row][q] and *inl is the slot's query, which the launch takes as its parameter block
 * -- the query reaches the GPU with the launch, with no copy queued ahead of it -- while the
 * kernel reads the new row through the slot's device mapping (k_new / v_new may already be the
 * slot's own rows: a deferred append).  *inl = NULL when any input is device memory
 * (stage_inputs then).  1 on success, else 0 with the error set. */
static int inline_inputs(tyb_cache *t, int layer, const float *q, const float *k_new, const float *v_new,
                         const float **inl, const char *what)
{
    *inl = NULL;
    const int rq = tyb_is_device_ptr(q);
    const int rk = k_new ? tyb_is_device_ptr(k_new) : 0, rv = v_new ? tyb_is_device_ptr(v_new) : 0;
    if (rq < 0 || rk < 0 || rv < 0) return 0;
    if (rq || rk || rv) return 1;
    if (!tyb_slots_ready(t, what)) return 0;
    float *slot = tyb_row_slot(t, layer);
    /* an earlier launch may still read the slot through its mapping (a deferred row's write) */
    if (!tyb_slot_wait(t, layer, what)) return 0;
    if (k_new && k_new != slot) memcpy(slot, k_new, TYB_ROW_FLOATS * sizeof(float));
    if (v_new && v_new != slot + TYB_ROW_FLOATS) memcpy(slot + TYB_ROW_FLOATS, v_new, TYB_ROW_FLOATS * sizeof(float));
    memcpy(slot + 2 * TYB_ROW_FLOATS, q, TYB_Q_FLOATS * sizeof(float));
    *inl = slot + 2 * TYB_ROW_FLOATS;
    return 1;
}

/* A host output of a one-sequence decode call, `n` floats: stored by the kernel through a device
 * mapping -- the caller's page-locked buffer in place, a pageable one by way of the cache's
 * page-locked staging (copied out after the wait) -- and marked unwritten first, so the call
 * can wait for the words themselves (tyb_wait_output).  Sets *dout (the device view) and *hout
 * (the host side the call waits on); 1 on success. */
static int host_output(tyb_cache *t, float *output, float *dout_mapped, int kind, size_t n, float **dout,
                       float **hout, const char *what)
{
    if (!tyb_slots_ready(t, what)) return 0;
    *hout = kind == TYB_MEM_PINNED ? output : t->h_out;
    *dout = kind == TYB_MEM_PINNED ? dout_mapped : t->h_out_dev;
    tyb_mark_unwritten(*hout, n);
    return 1;
}

/* The single-token inputs of a decode call -- q [16][128] and, for an append, k_new / v_new
 * [8][128] (NULL when absent) -- on the device, when they cannot all travel as the launch's
 * parameter block (inline_inputs: some are device memory, some host memory, or the output is
 * gathered from every rank).  Device buffers are used in place.  Host buffers (page-locked or
 * not) are copied now into the layer's page-locked slot of the cache, so the caller may reuse
 * them on return, and the slot reaches the device in ONE copy, into the cache's staging area,
 * ahead of the kernel: the splits then read L2 instead of each fetching the query over the bus.
 * k_new / v_new may already be the slot's own rows (a deferred append).
 * 1 on success, else 0 with the error set. */
static int stage_inputs(tyb_cache *t, int layer, const float *q, const float *k_new, const float *v_new,
                        const float **dq, const float **dk, const float **dv, void *st, const char *what)
{
    const int rq = tyb_is_device_ptr(q);
    const int rk = k_new ? tyb_is_device_ptr(k_new) : 1, rv = v_new ? tyb_is_device_ptr(v_new) : 1;
    if (rq < 0 || rk < 0 || rv < 0) return 0;
    *dq = q;
    *dk = k_new;
    *dv = v_new;
    if (rq && rk && rv) return 1;
    if (!tyb_slots_ready(t, what)) return 0;
    float *slot = tyb_row_slot(t, layer);
    /* the slot's previous contents have been read (a deferred row is already in place) */
    if (!tyb_slot_wait(t, layer, what)) return 0;
    if (!rk && k_new != slot) memcpy(slot, k_new, TYB_ROW_FLOATS * sizeof(float));
    if (!rv && v_new != slot + TYB_ROW_FLOATS) memcpy(slot + TYB_ROW_FLOATS, v_new, TYB_ROW_FLOATS * sizeof(float));
    if (!rq) memcpy(slot + 2 * TYB_ROW_FLOATS, q, TYB_Q_FLOATS * sizeof(float));
    const size_t lo = (!rk || !rv) ? 0 : 2 * TYB_ROW_FLOATS, hi = !rq ? TYB_SLOT_FLOATS : 2 * TYB_ROW_FLOATS;
    float *stage = t->d_kv_stage; /* >= 16 KB */
    if (!tyb_cuda_ok(cudaMemcpyAsync(stage + lo, slot + lo, (hi - lo) * sizeof(float), cudaMemcpyHostToDevice,
                                     (cudaStream_t)st),
                     what) ||
        !tyb_slot_consumed(t, layer, st, what))
        return 0;
    if (!rq) *dq = stage + 2 * TYB_ROW_FLOATS;
    if (!rk) *dk = stage;
    if (!rv) *dv = stage + TYB_ROW_FLOATS;
    return 1;
}

void attention_decode_gqa(const float *q, const KVCache *cache, float *output, int layer_idx,
                          int kv_len, float scale)
{
    const char *what = "attention_decode_gqa";
    tyb_cache *t = tyb_cache_from(cache);
    if (!t || !check_layer(layer_idx, what)) return;
    if (!q || !output) {
        tyb_set_error("%s: NULL q/output", what);
        return;
    }
    if (kv_len < 0 || kv_len > cache->max_seq_len) {
        tyb_set_error("%s: kv_len %d out of range [0, %d]", what, kv_len, cache->max_seq_len);
        return;
    }
    if (t->pending[layer_idx] >= 0 && t->pending[layer_idx] == kv_len - 1) {
        /* The row kv_cache_append staged for this layer is the last one attended: append and
         * attend in one launch (kernel/decoder.c:96-105), the row taken from its slot. */
        const float *slot = tyb_row_slot(t, layer_idx);
        t->pending[layer_idx] = -1;
        decode_append_impl(q, slot, slot + TYB_ROW_FLOATS, (KVCache *)cache, output, layer_idx, scale, 0,
                           KV_NUM_KV_HEADS, NULL, kv_len - 1, what);
        return;
    }
    if (!tyb_flush_pending(t, layer_idx, what)) return;
    void *st = tyb_stream();
    int ok = 0;
    const float *inl = NULL, *dq = q, *unused_k, *unused_v;
    float *hout = NULL;
    if (kv_len > 0 && !inline_inputs(t, layer_idx, q, NULL, NULL, &inl, what)) return;
    if (kv_len > 0 && !inl && !stage_inputs(t, layer_idx, q, NULL, NULL, &dq, &unused_k, &unused_v, st, what))
        return;
    float *dout = small_view(output, NULL, 0, &ok, st, what);
    if (ok < 0 || (ok != TYB_MEM_HOST && !dout)) return;
    if (kv_len > 0 && ok != TYB_MEM_DEVICE) {
        if (!host_output(t, output, dout, ok, TYB_Q_FLOATS, &dout, &hout, what)) return;
    } else if (ok == TYB_MEM_HOST) {
        dout = t->d_out;
    }
    if (kv_len == 0) {
        /* The reference's loops do not run and the output stays zeroed (:186-190). */
        if (ok == TYB_MEM_PINNED) {
            memset(output, 0, TYB_Q_FLOATS * sizeof(float));
            dout = NULL;
        } else if (!tyb_cuda_ok(cudaMemsetAsync(dout, 0, TYB_Q_FLOATS * sizeof(float), (cudaStream_t)st), what)) {
            return;
        }
    } else {
        const tyb_seq_kv one = tyb_layer_rows(t, layer_idx, kv_len);
        const int early = tyb_prefetch_rows(cache, layer_idx, kv_len);
        if (!tyb_cuda_ok(decode_launch(dq, dout, NULL, one, 1, kv_len, t->dtype, scale, early, t->d_partials,
                                       t->d_counters, TYB_DEC_DEVICE_SMALL | TYB_DEC_WIDE_COUNTERS, inl, st),
                         what))
            return;
        tyb_note_nowrite(st);
        if (hout) {
            /* host output: wait for its words, not for the launch */
            if (tyb_wait_output(hout, TYB_Q_FLOATS, st, what) && ok == TYB_MEM_HOST)
                memcpy(output, t->h_out, TYB_Q_FLOATS * sizeof(float));
            return;
        }
    }
    if (ok == TYB_MEM_HOST) {
        if (!tyb_cuda_ok(cudaMemcpyAsync(output, dout, TYB_Q_FLOATS * sizeof(float), cudaMemcpyDeviceToHost,
                                         (cudaStream_t)st),
                         what))
            return;
    }
    /* A host output (pageable or page-locked): the call returns once the result is there. */
    if (ok != TYB_MEM_DEVICE) tyb_finish(st, what);
}

/* ---- pipelined drop-in prefill from host buffers ----------------------------------------
 * kernel/decoder.c:106-117 calls attention_prefill_gqa with host q/k/v/output: 64 MB in and 32 MB
 * out per 4K-token layer over PCIe, against ~0.25 ms of tensor-core work.  Done in order, the
 * call is three copies, the kernels, then the copy back.  Here the rows go in chunks (multiples
 * of the 128-row query tile): chunk c's queries and K/V rows are copied in on one stream while
 * chunk c - 1 is split and attended (causal: its queries see only rows up to its own) on the
 * library's stream, and its output rows go back on a third stream -- the inbound and outbound
 * copies overlap each other and the kernels.  The output of a chunk is written over its staged
 * queries (each query tile is read before its output is written, by the same CTA), so the
 * staging needs no more room than the serial path.  Streams and events: per thread and device,
 * made on first use and kept until exit. */
#define TYB_PIPE_DEVICES 64
static _Thread_local cudaStream_t g_pipe_in[TYB_PIPE_DEVICES], g_pipe_out[TYB_PIPE_DEVICES];
static _Thread_local cudaEvent_t g_pipe_ev[TYB_PIPE_DEVICES][4]; /* start, in, done, out */

static int pipe_ready(int dev, const char *what)
{
    if (g_pipe_in[dev]) return 1;
    cudaStream_t a = NULL, b = NULL;
    cudaEvent_t e[4] = {NULL, NULL, NULL, NULL};
    int ok = tyb_cuda_ok(cudaStreamCreateWithFlags(&a, cudaStreamNonBlocking), what) &&
             tyb_cuda_ok(cudaStreamCreateWithFlags(&b, cudaStreamNonBlocking), what);
    for (int i = 0; ok && i < 4; i++) ok = tyb_cuda_ok(cudaEventCreateWithFlags(&e[i], cudaEventDisableTiming), what);
    if (!ok) {
        if (a) cudaStreamDestroy(a);
        if (b) cudaStreamDestroy(b);
        for (int i = 0; i < 4; i++)
            if (e[i]) cudaEventDestroy(e[i]);
        return 0;
    }
    g_pipe_out[dev] = b;
    for (int i = 0; i < 4; i++) g_pipe_ev[dev][i] = e[i];
    g_pipe_in[dev] = a;
    return 1;
}

/* q/k/v/output host buffers of S rows (S keys), sq: device staging of the queries (>= S rows),
 * so: of the raw K then V rows (2 x S rows), ksp / vsp: the hi|lo BF16 pairs.  1 on success. */
static int prefill_pipelined(const float *q, const float *k, const float *v, float *output, int S, float scale,
                             float *sq, float *so, unsigned char *ksp, unsigned char *vsp, void *st, const char *what)
{
    int dev = 0;
    if (!tyb_cuda_ok(cudaGetDevice(&dev), what)) return 0;
    if (dev < 0 || dev >= TYB_PIPE_DEVICES) {
        tyb_set_error("%s: device %d out of range", what, dev);
        return 0;
    }
    if (!pipe_ready(dev, what)) return 0;
    cudaStream_t in = g_pipe_in[dev], out = g_pipe_out[dev], cs = (cudaStream_t)st;
    cudaEvent_t *ev = g_pipe_ev[dev];
    const size_t kb = (size_t)S * TYB_ROW_FLOATS * sizeof(float);
    /* about eight chunks, at least 512 rows each, whole query tiles */
    int chunk = ((S + 7) / 8 + 127) / 128 * 128;
    if (chunk < 512) chunk = 512;
    /* Both copy streams start after the work already queued on the library's stream. */
    int ok = tyb_cuda_ok(cudaEventRecord(ev[0], cs), what) && tyb_cuda_ok(cudaStreamWaitEvent(in, ev[0], 0), what) &&
             tyb_cuda_ok(cudaStreamWaitEvent(out, ev[0], 0), what);
    for (int r0 = 0; ok && r0 < S; r0 += chunk) {
        const int n = S - r0 < chunk ? S - r0 : chunk;
        const size_t qo = (size_t)r0 * TYB_Q_FLOATS, ko = (size_t)r0 * TYB_ROW_FLOATS;
        const size_t qn = (size_t)n * TYB_Q_FLOATS * sizeof(float), kn = (size_t)n * TYB_ROW_FLOATS * sizeof(float);
        float *sk = so + ko, *sv = so + kb / sizeof(float) + ko;
        ok = tyb_cuda_ok(cudaMemcpyAsync(sk, k + ko, kn, cudaMemcpyHostToDevice, in), what) &&
             tyb_cuda_ok(cudaMemcpyAsync(sv, v + ko, kn, cudaMemcpyHostToDevice, in), what) &&
             tyb_cuda_ok(cudaMemcpyAsync(sq + qo, q + qo, qn, cudaMemcpyHostToDevice, in), what) &&
             tyb_cuda_ok(cudaEventRecord(ev[1], in), what) && tyb_cuda_ok(cudaStreamWaitEvent(cs, ev[1], 0), what) &&
             tyb_cuda_ok(tyb_kv_split_rows_launch(sk, sv, TYB_ROW_FLOATS, KV_HEAD_DIM, n, r0, S, ksp, ksp + kb / 2, vsp,
                                                  vsp + kb / 2, st),
                         what) &&
             tyb_cuda_ok(tyb_prefill_tc32_launch(sq + qo, sq + qo, n, r0, r0 + n, ksp, ksp + kb / 2, vsp, vsp + kb / 2, S,
                                                 scale, st),
                         what) &&
             tyb_cuda_ok(cudaEventRecord(ev[2], cs), what) && tyb_cuda_ok(cudaStreamWaitEvent(out, ev[2], 0), what) &&
             tyb_cuda_ok(cudaMemcpyAsync(output + qo, sq + qo, qn, cudaMemcpyDeviceToHost, out), what);
    }
    /* The library's stream resumes after the last copy back (later work may reuse the staging). */
    const int joined = tyb_cuda_ok(cudaEventRecord(ev[3], out), what) &&
                       tyb_cuda_ok(cudaStreamWaitEvent(cs, ev[3], 0), what);
    if (!ok || !joined) {
        /* nothing queued may outlive the call: the copies name the caller's buffers */
        cudaStreamSynchronize(in);
        cudaStreamSynchronize(out);
        return 0;
    }
    tyb_note_nowrite(st);
    return tyb_finish(st, what);
}

void attention_prefill_gqa(const float *q, const float *k, const float *v, float *output, int Sq,
                           int Sk, float scale, float *q_hm, float *k_hm, float *v_hm, float *o_hm)
{
    const char *what = "attention_prefill_gqa";
    if (Sq < 0 || Sk < 0) {
        tyb_set_error("%s: negative Sq/Sk (%d, %d)", what, Sq, Sk);
        return;
    }
    if (Sq == 0) return;
    if (!q || !output) {
        tyb_set_error("%s: NULL q/output", what);
        return;
    }
    /* Keys visible to any query are rows < min(Sk, Sq) (mask k_pos > q_pos, :293). */
    const int kv_rows = Sk < Sq ? Sk : Sq;
    if (kv_rows > 0 && (!k || !v)) {
        tyb_set_error("%s: NULL k/v", what);
        return;
    }
    void *st = tyb_stream();
    const size_t qb = (size_t)Sq * TYB_Q_FLOATS * sizeof(float);
    const size_t kb = (size_t)kv_rows * TYB_ROW_FLOATS * sizeof(float); /* = bytes of its hi|lo BF16 pair */

    int qd = tyb_is_device_ptr(q), od = tyb_is_device_ptr(output);
    int kd = kv_rows ? tyb_is_device_ptr(k) : 1, vd = kv_rows ? tyb_is_device_ptr(v) : 1;
    if (qd < 0 || kd < 0 || vd < 0 || od < 0) return;
    if (kv_rows == 0) {
        /* No key at all: every row's sum is 0 and the reference writes zeros (:347-361). */
        if (!od) {
            memset(output, 0, qb);
            return;
        }
        tyb_cuda_ok(cudaMemsetAsync(output, 0, qb, (cudaStream_t)st), what);
        return;
    }
    /* The scratch's device slots (kernel/scratch.h q_hm..o_hm, sized by max_seq_len) hold all
     * the staging when the caller passes them, as kernel/decoder.c:113-117 does: q_hm the queries
     * of a host q; k_hm / v_hm the BF16 hi|lo pairs of K / V; o_hm the FP32 rows of a host K and V
     * on their way to the split, then the output of a host `output` (the split has consumed the
     * rows by then: the attention kernel waits for it).  Otherwise the library's workspace. */
    const size_t kv_stage = (kd ? 0 : kb) + (vd ? 0 : kb);
    const size_t o_stage = (!od && qb > kv_stage) ? qb : kv_stage;
    float *sq = NULL, *so = NULL;
    if (!qd) sq = (q_hm && tyb_registry_size(q_hm) >= qb) ? q_hm : (float *)tyb_workspace(TYB_WS_Q, qb);
    unsigned char *ksp = (k_hm && tyb_registry_size(k_hm) >= kb) ? (unsigned char *)k_hm
                                                               : (unsigned char *)tyb_workspace(TYB_WS_K, kb);
    unsigned char *vsp = (v_hm && tyb_registry_size(v_hm) >= kb) ? (unsigned char *)v_hm
                                                               : (unsigned char *)tyb_workspace(TYB_WS_V, kb);
    if (o_stage) so = (o_hm && tyb_registry_size(o_hm) >= o_stage) ? o_hm : (float *)tyb_workspace(TYB_WS_OUT, o_stage);
    if ((!qd && !sq) || !ksp || !vsp || (o_stage && !so)) return;

    /* All four in host memory and every query row seeing its own key (Sk >= Sq): chunks of rows
     * stream in and out while the kernels run (prefill_pipelined). */
    if (!qd && !kd && !vd && !od && kv_rows == Sq && Sq >= 2 * 512 && sq) {
        prefill_pipelined(q, k, v, output, Sq, scale, sq, so, ksp, vsp, st, what);
        return;
    }
    const float *dq = to_device(q, sq, qb, &qd, st, what);
    const float *dk = to_device(k, so, kb, &kd, st, what);
    const float *dv = dk ? to_device(v, so + (kd ? 0 : kb / sizeof(float)), kb, &vd, st, what) : NULL;
    if (!dq || !dk || !dv) return;
    float *dout = od ? output : so;
    /* Token-major rows: row stride 8 x 128, head stride 128 (:27-30). */
    if (!tyb_cuda_ok(tyb_kv_split_launch(dk, dv, TYB_ROW_FLOATS, KV_HEAD_DIM, kv_rows, ksp, ksp + kb / 2, vsp,
                                         vsp + kb / 2, st),
                     what) ||
        !tyb_cuda_ok(tyb_prefill_tc32_launch(dq, dout, Sq, 0, kv_rows, ksp, ksp + kb / 2, vsp, vsp + kb / 2, kv_rows,
                                             scale, st),
                     what))
        return;
    tyb_note_nowrite(st);
    if (!od && !tyb_cuda_ok(cudaMemcpyAsync(output, dout, qb, cudaMemcpyDeviceToHost, (cudaStream_t)st), what))
        return;
    if (!qd || !kd || !vd || !od) tyb_finish(st, what);
}

void attention_chunked_prefill_gqa(const float *q, const KVCache *cache, float *output,
                                   int layer_idx, int chunk_len, int pos_offset, float scale)
{
    const char *what = "attention_chunked_prefill_gqa";
    tyb_cache *t = tyb_cache_from(cache);
    if (!t || !check_layer(layer_idx, what)) return;
    if (chunk_len < 0 || pos_offset < 0 || pos_offset + chunk_len > cache->max_seq_len) {
        tyb_set_error("%s: rows [%d, %d) exceed max_seq_len %d", what, pos_offset, pos_offset + chunk_len,
                      cache->max_seq_len);
        return;
    }
    if (chunk_len == 0) return;
    if (!q || !output) {
        tyb_set_error("%s: NULL q/output", what);
        return;
    }
    if (!tyb_flush_pending(t, layer_idx, what)) return;
    void *st = tyb_stream();
    const size_t qb = (size_t)chunk_len * TYB_Q_FLOATS * sizeof(float);
    int qd = tyb_is_device_ptr(q), od = tyb_is_device_ptr(output);
    if (qd < 0 || od < 0) return;
    float *sq = qd ? NULL : (float *)tyb_workspace(TYB_WS_Q, qb);
    float *so = od ? NULL : (float *)tyb_workspace(TYB_WS_OUT, qb);
    if ((!qd && !sq) || (!od && !so)) return;
    const float *dq = to_device(q, sq, qb, &qd, st, what);
    if (!dq) return;
    float *dout = od ? output : so;
    const void *kl = tyb_slab_head(t, t->k_slab, layer_idx, 0);
    const void *vl = tyb_slab_head(t, t->v_slab, layer_idx, 0);
    const int total = pos_offset + chunk_len; /* keys of query i: rows <= pos_offset + i (:443-459) */
    int rc;
    if (t->dtype == TYB_BF16) {
        /* BF16 rows are exact as BF16 operands (lo = 0): the tiles come straight from the cache. */
        rc = tyb_prefill_tc32_launch(dq, dout, chunk_len, pos_offset, total, kl, NULL, vl, NULL, cache->max_seq_len,
                                     scale, st);
    } else {
        /* FP32 rows: split rows [0, total) of the layer (head-first: row stride 128, head stride
         * max_seq x 128, :425-427) into hi|lo pairs in the cache's staging area, which holds
         * 8 KB per row of max_seq_len (K hi, K lo, V hi, V lo at 2 KB per row each). */
        unsigned char *sp = (unsigned char *)t->d_kv_stage;
        const size_t part = (size_t)total * TYB_ROW_FLOATS * 2;
        rc = tyb_kv_split_launch((const float *)kl, (const float *)vl, KV_HEAD_DIM,
                                 (long long)cache->max_seq_len * KV_HEAD_DIM, total, sp, sp + part, sp + 2 * part,
                                 sp + 3 * part, st);
        if (rc == 0)
            rc = tyb_prefill_tc32_launch(dq, dout, chunk_len, pos_offset, total, sp, sp + part, sp + 2 * part,
                                         sp + 3 * part, total, scale, st);
    }
    if (!tyb_cuda_ok(rc, what)) return;
    tyb_note_nowrite(st);
    if (!od && !tyb_cuda_ok(cudaMemcpyAsync(output, dout, qb, cudaMemcpyDeviceToHost, (cudaStream_t)st), what))
        return;
    if (!qd || !od) tyb_finish(st, what);
}

int attention_decode_gqa_batched(const float *q, const KVCache *const *caches, const int *kv_lens,
                                 float *output, int batch, int layer_idx, float scale)
{
    const char *what = "attention_decode_gqa_batched";
    if (batch <= 0 || !caches || !kv_lens || !q || !output) {
        tyb_set_error("%s: need batch > 0 and non-NULL q/caches/kv_lens/output", what);
        return 1;
    }
    if (!check_layer(layer_idx, what)) return 1;
    tyb_seq_kv *descs = (tyb_seq_kv *)malloc(sizeof(tyb_seq_kv) * (size_t)batch);
    if (!descs) {
        tyb_set_error("%s: out of host memory", what);
        return 1;
    }
    int dtype = -1, max_kv = 0, ok = 1;
    for (int b = 0; b < batch && ok; b++) {
        tyb_cache *t = tyb_cache_from(caches[b]);
        if (!t || !tyb_flush_pending(t, layer_idx, what)) { ok = 0; break; }
        if (dtype >= 0 && t->dtype != dtype) {
            tyb_set_error("%s: caches mix element types", what);
            ok = 0;
            break;
        }
        dtype = t->dtype;
        if (kv_lens[b] < 1 || kv_lens[b] > t->pub.max_seq_len) {
            tyb_set_error("%s: kv_lens[%d] = %d out of range [1, %d]", what, b, kv_lens[b], t->pub.max_seq_len);
            ok = 0;
            break;
        }
        descs[b].k = tyb_slab_head(t, t->k_slab, layer_idx, 0);
        descs[b].v = tyb_slab_head(t, t->v_slab, layer_idx, 0);
        descs[b].kv_len = kv_lens[b];
        descs[b].row_capacity = t->pub.max_seq_len;
        descs[b].pf_k = descs[b].pf_v = NULL;
        if (kv_lens[b] > max_kv) max_kv = kv_lens[b];
    }
    if (!ok) {
        free(descs);
        return 1;
    }
    void *st = tyb_stream();
    const size_t qb = (size_t)batch * TYB_Q_FLOATS * sizeof(float);
    /* Descriptors (and, for BF16 caches, two tensor maps per sequence ahead of them). */
    const size_t desc_bytes = sizeof(tyb_seq_kv) * (size_t)batch;
    const size_t upload_bytes = (dtype == TYB_BF16 ? tyb_decode_maps_bytes(batch) : 0) + desc_bytes;
    unsigned char *upload = (unsigned char *)tyb_workspace(TYB_WS_DESC, upload_bytes);
    tyb_seq_kv *ddesc = upload ? (tyb_seq_kv *)(upload + (upload_bytes - desc_bytes)) : NULL;
    int qd = tyb_is_device_ptr(q), od = tyb_is_device_ptr(output);
    float *sq = (qd == 0) ? (float *)tyb_workspace(TYB_WS_Q, qb) : NULL;
    float *so = (od == 0) ? (float *)tyb_workspace(TYB_WS_OUT, qb) : NULL;
    if (!ddesc || qd < 0 || od < 0 || (!qd && !sq) || (!od && !so)) {
        free(descs);
        return 1;
    }
    int chunk, nsplit;
    tyb_decode_plan(batch, max_kv, dtype, &chunk, &nsplit);
    float *part = (float *)tyb_workspace(TYB_WS_PARTIALS, tyb_decode_partial_floats(batch, nsplit) * sizeof(float));
    unsigned int *cnt =
        (unsigned int *)tyb_workspace(TYB_WS_COUNTERS, sizeof(unsigned int) * (size_t)batch * KV_NUM_KV_HEADS);
    const float *dq = (part && cnt) ? to_device(q, sq, qb, &qd, st, what) : NULL;
    if (!dq) {
        free(descs);
        return 1;
    }
    float *dout = od ? output : so;
    if (dtype == TYB_BF16) {
        /* Uploads the tensor maps and the descriptors in one copy, then launches. */
        ok = tyb_cuda_ok(tyb_decode_launch_batched(dq, dout, descs, upload, batch, max_kv, scale, part, cnt, st), what);
        free(descs);
        if (!ok) return 1;
    } else {
        /* The descriptor upload reads host memory: pageable copies are staged by the driver
         * before cudaMemcpyAsync returns, so `descs` can be freed right after. */
        ok = tyb_cuda_ok(cudaMemcpyAsync(ddesc, descs, desc_bytes, cudaMemcpyHostToDevice, (cudaStream_t)st), what);
        free(descs);
        if (!ok) return 1;
        tyb_seq_kv none;
        memset(&none, 0, sizeof none);
        if (!tyb_cuda_ok(decode_launch(dq, dout, ddesc, none, batch, max_kv, dtype, scale, 0, part, cnt,
                                       TYB_DEC_DEVICE_SMALL, NULL, st),
                         what))
            return 1;
    }
    tyb_note_nowrite(st);
    if (!od && !tyb_cuda_ok(cudaMemcpyAsync(output, dout, qb, cudaMemcpyDeviceToHost, (cudaStream_t)st), what))
        return 1;
    if (!qd || !od) return tyb_finish(st, what) ? 0 : 1;
    return 0;
}

/* gather: NULL, or the connected output gather (the output is then the whole [16][128],
 * assembled from every rank's shard; see attn_gather_init). */
/* pos_at: the row the new K/V go to, kv_len = pos_at + 1; -1 for cache->seq_len (then a deferred
 * row of the layer is written first; >= 0 is the consumption of that row, staged by the caller). */
static int decode_append_impl(const float *q, const float *k_new, const float *v_new, KVCache *cache, float *output,
                              int layer_idx, float scale, int kvh0, int nkvh, const void *gather, int pos_at,
                              const char *what)
{
    tyb_cache *t = tyb_cache_from(cache);
    if (!t || !check_layer(layer_idx, what)) return 1;
    if (!q || !k_new || !v_new || !output) {
        tyb_set_error("%s: NULL q/k_new/v_new/output", what);
        return 1;
    }
    if (pos_at < 0 && !tyb_flush_pending(t, layer_idx, what)) return 1;
    const int pos = pos_at >= 0 ? pos_at : cache->seq_len;
    if (pos < 0 || pos >= cache->max_seq_len) {
        tyb_set_error("%s: row %d exceeds max_seq_len %d", what, pos, cache->max_seq_len);
        return 1;
    }
    void *st = tyb_stream();
    int ok = 0;
    const float *inl = NULL, *dq = q, *dk = k_new, *dv = v_new;
    float *hout = NULL;
    int flags = TYB_DEC_DEVICE_SMALL | TYB_DEC_WIDE_COUNTERS;
    if (!gather && !inline_inputs(t, layer_idx, q, k_new, v_new, &inl, what)) return 1;
    if (!inl && !stage_inputs(t, layer_idx, q, k_new, v_new, &dq, &dk, &dv, st, what)) return 1;
    float *dout = small_view(output, NULL, 0, &ok, st, what);
    /* rows of the query heads computed (all 16 when gathered from every rank) */
    const size_t out_floats = (size_t)2 * (gather ? KV_NUM_KV_HEADS : nkvh) * KV_HEAD_DIM;
    if (ok < 0 || (ok != TYB_MEM_HOST && !dout)) return 1;
    if (!gather && ok != TYB_MEM_DEVICE) {
        if (!host_output(t, output, dout, ok, out_floats, &dout, &hout, what)) return 1;
    } else if (ok == TYB_MEM_HOST) {
        dout = t->d_out;
    }
    if (inl && hout) {
        /* a blocking call: the query as the parameter block, the new row read through the slot's
         * device mapping (the output is written after it is read, so the slot is free on return) */
        const float *slot_dev = t->h_rows_dev + (size_t)layer_idx * TYB_SLOT_FLOATS;
        dk = slot_dev;
        dv = slot_dev + TYB_ROW_FLOATS;
    } else if (inl) {
        /* returns before the kernel runs: the whole slot as the parameter block (nothing on the
         * device reads the slot, so the host may rewrite it at once) */
        inl -= 2 * TYB_ROW_FLOATS;
        flags |= TYB_DEC_INLINE_ROW;
    }
    const tyb_seq_kv one = tyb_layer_rows(t, layer_idx, pos + 1);
    const int early = tyb_prefetch_rows(cache, layer_idx, pos);
    if (!tyb_cuda_ok(tyb_decode_launch_heads(dq, dout, NULL, one, 1, pos + 1, t->dtype, scale, t->d_partials,
                                             t->d_counters, dk, dv, early, kvh0, nkvh, flags, gather, inl, st),
                     what))
        return 1;
    tyb_note_write(cache, layer_idx, pos, st);
    if (hout) {
        /* host output: wait for its words, not for the launch */
        if (!tyb_wait_output(hout, out_floats, st, what)) return 1;
        if (ok == TYB_MEM_HOST) memcpy(output, t->h_out, out_floats * sizeof(float));
        return 0;
    }
    if (ok == TYB_MEM_HOST && !tyb_cuda_ok(cudaMemcpyAsync(output, dout, out_floats * sizeof(float),
                                                           cudaMemcpyDeviceToHost, (cudaStream_t)st),
                                           what))
        return 1;
    /* A host output (pageable or page-locked): the call returns once the result is there.  Host
     * inputs were copied before the launch (stage_inputs), so they need no wait. */
    if (ok != TYB_MEM_DEVICE) return tyb_finish(st, what) ? 0 : 1;
    return 0;
}

int attention_decode_append_gqa(const float *q, const float *k_new, const float *v_new, KVCache *cache,
                                float *output, int layer_idx, float scale)
{
    return decode_append_impl(q, k_new, v_new, cache, output, layer_idx, scale, 0, KV_NUM_KV_HEADS, NULL, -1,
                              "attention_decode_append_gqa");
}

static int check_heads(int kv_head0, int kv_heads, const char *what)
{
    if (kv_heads < 1 || kv_head0 < 0 || kv_head0 + kv_heads > KV_NUM_KV_HEADS) {
        tyb_set_error("%s: KV heads [%d, %d) outside [0, %d)", what, kv_head0, kv_head0 + kv_heads, KV_NUM_KV_HEADS);
        return 0;
    }
    return 1;
}

int attention_decode_append_gqa_heads(const float *q, const float *k_new, const float *v_new, KVCache *cache,
                                      float *output, int layer_idx, float scale, int kv_head0, int kv_heads)
{
    const char *what = "attention_decode_append_gqa_heads";
    if (!check_heads(kv_head0, kv_heads, what)) return 1;
    return decode_append_impl(q, k_new, v_new, cache, output, layer_idx, scale, kv_head0, kv_heads, NULL, -1, what);
}

int attn_gather_init(int rank, int world)
{
    if (world < 1 || world > 8 || rank < 0 || rank >= world) {
        tyb_set_error("attn_gather_init: need 0 <= rank (%d) < world (%d) <= 8", rank, world);
        return 1;
    }
    return tyb_cuda_ok(tyb_gather_init(rank, world), "attn_gather_init") ? 0 : 1;
}

int attn_gather_handle(void *handle_out)
{
    return tyb_cuda_ok(tyb_gather_handle(handle_out), "attn_gather_handle") ? 0 : 1;
}

int attn_gather_connect(const void *handles)
{
    return tyb_cuda_ok(tyb_gather_connect(handles), "attn_gather_connect") ? 0 : 1;
}

void attn_gather_close(void) { tyb_gather_close(); }

int attention_decode_append_gqa_gathered(const float *q, const float *k_new, const float *v_new, KVCache *cache,
                                         float *output, int layer_idx, float scale, int kv_head0, int kv_heads)
{
    const char *what = "attention_decode_append_gqa_gathered";
    if (!check_heads(kv_head0, kv_heads, what)) return 1;
    int world = 0, rank = 0;
    const void *g = tyb_gather_dev(&world, &rank);
    if (!g) {
        tyb_set_error("%s: no connected output gather (attn_gather_init / attn_gather_connect)", what);
        return 1;
    }
    tyb_cache *t = tyb_cache_from(cache);
    if (t && t->dtype != TYB_BF16) {
        tyb_set_error("%s: the cache must hold BF16 rows", what);
        return 1;
    }
    return decode_append_impl(q, k_new, v_new, cache, output, layer_idx, scale, kv_head0, kv_heads, g, -1, what);
}

int attention_decode_append_fused_gqa(const float *q_raw, const float *k_raw, const float *v_new,
                                      const float *q_norm, const float *k_norm, const float *token_cos,
                                      const float *token_sin, KVCache *cache, float *output, int layer_idx,
                                      float scale, float eps)
{
    const char *what = "attention_decode_append_fused_gqa";
    tyb_cache *t = tyb_cache_from(cache);
    if (!t || !check_layer(layer_idx, what)) return 1;
    if (t->dtype != TYB_BF16) {
        tyb_set_error("%s: the cache must hold BF16 rows (kv_cache_alloc_ex(.., ATTN_KV_BF16))", what);
        return 1;
    }
    const int pos = cache->seq_len;
    if (pos < 0 || pos >= cache->max_seq_len) {
        tyb_set_error("%s: row %d exceeds max_seq_len %d", what, pos, cache->max_seq_len);
        return 1;
    }
    if (!tyb_flush_pending(t, layer_idx, what)) return 1;
    const void *ptrs[8] = {q_raw, k_raw, v_new, q_norm, k_norm, token_cos, token_sin, output};
    for (int i = 0; i < 8; i++) {
        const int d = ptrs[i] ? tyb_is_device_ptr(ptrs[i]) : 0;
        if (d < 0) return 1;
        if (!d) {
            tyb_set_error("%s: argument %d must be device memory", what, i);
            return 1;
        }
        if (!tyb_aligned16(ptrs[i], what)) return 1;
    }
    void *st = tyb_stream();
    const tyb_seq_kv one = tyb_layer_rows(t, layer_idx, pos + 1);
    const int early = tyb_prefetch_rows(cache, layer_idx, pos);
    tyb_qk_prep prep;
    prep.q_norm = q_norm;
    prep.k_norm = k_norm;
    prep.cos = token_cos;
    prep.sin = token_sin;
    prep.eps = eps;
    if (!tyb_cuda_ok(tyb_decode_launch_fused(q_raw, output, one, pos + 1, scale, t->d_partials, t->d_counters, k_raw,
                                             v_new, early, &prep, st),
                     what))
        return 1;
    tyb_note_write(cache, layer_idx, pos, st);
    return 0;
}

/* xchg_dev / xchg_maps / epoch: the sharded form (tyb_prefill_sharded); NULL / NULL / 0 otherwise. */
static int prefill_fused_impl(const void *q_raw, const void *k_raw, const void *v_raw, int in_dtype,
                              const float *q_norm, const float *k_norm, const float *token_cos, const float *token_sin,
                              KVCache *cache, int layer_idx, void *output, int out_dtype, int seq_len, float scale,
                              float eps, int kvh0, int nkvh, int head_major, const tyb_prefill_x *xchg_dev,
                              const void *xchg_maps, unsigned int epoch, const char *what)
{
    tyb_cache *t = tyb_cache_from(cache);
    if (!t || !check_layer(layer_idx, what)) return 1;
    if (t->dtype != TYB_BF16) {
        tyb_set_error("%s: the cache must hold BF16 rows (kv_cache_alloc_ex(.., ATTN_KV_BF16))", what);
        return 1;
    }
    if ((in_dtype != ATTN_DT_F32 && in_dtype != ATTN_DT_BF16) || (out_dtype != ATTN_DT_F32 && out_dtype != ATTN_DT_BF16)) {
        tyb_set_error("%s: unknown element type", what);
        return 1;
    }
    const int pos0 = cache->seq_len;
    if (seq_len < 0 || pos0 < 0 || pos0 + seq_len > cache->max_seq_len) {
        tyb_set_error("%s: rows [%d, %d) exceed max_seq_len %d", what, pos0, pos0 + seq_len, cache->max_seq_len);
        return 1;
    }
    if (seq_len == 0) return 0;
    if (!tyb_flush_pending(t, layer_idx, what)) return 1;
    const void *ptrs[9] = {q_raw, k_raw, v_raw, q_norm, k_norm, token_cos, token_sin, output, NULL};
    for (int i = 0; i < 8; i++) {
        const int d = ptrs[i] ? tyb_is_device_ptr(ptrs[i]) : 0;
        if (d < 0) return 1;
        if (!d) {
            tyb_set_error("%s: argument %d must be device memory", what, i);
            return 1;
        }
        if (!tyb_aligned16(ptrs[i], what)) return 1;
    }
    void *st = tyb_stream();
    void *kl = tyb_slab_head(t, t->k_slab, layer_idx, 0), *vl = tyb_slab_head(t, t->v_slab, layer_idx, 0);
    if (!tyb_cuda_ok(tyb_kv_prep_launch(k_raw, v_raw, in_dtype == ATTN_DT_BF16, k_norm, token_cos, token_sin, kl, vl,
                                        cache->max_seq_len, pos0, seq_len, eps, kvh0, nkvh, st),
                     what))
        return 1;
    tyb_note_write(cache, layer_idx, pos0, st);
    if (!tyb_cuda_ok(tyb_prefill_tc_launch(q_raw, in_dtype == ATTN_DT_BF16, q_norm, token_cos, token_sin, kl, vl,
                                           cache->max_seq_len, output, out_dtype == ATTN_DT_BF16, seq_len, pos0, scale,
                                           eps, kvh0, nkvh, head_major, xchg_dev, xchg_maps, epoch, st),
                     what))
        return 1;
    tyb_note_nowrite(st);
    return 0;
}

int attention_prefill_fused_gqa(const void *q_raw, const void *k_raw, const void *v_raw, int in_dtype,
                                const float *q_norm, const float *k_norm, const float *token_cos,
                                const float *token_sin, KVCache *cache, int layer_idx, void *output, int out_dtype,
                                int seq_len, float scale, float eps)
{
    return prefill_fused_impl(q_raw, k_raw, v_raw, in_dtype, q_norm, k_norm, token_cos, token_sin, cache, layer_idx,
                              output, out_dtype, seq_len, scale, eps, 0, KV_NUM_KV_HEADS, 0, NULL, NULL, 0,
                              "attention_prefill_fused_gqa");
}

int attention_prefill_fused_gqa_heads(const void *q_raw, const void *k_raw, const void *v_raw, int in_dtype,
                                      const float *q_norm, const float *k_norm, const float *token_cos,
                                      const float *token_sin, KVCache *cache, int layer_idx, void *output,
                                      int out_dtype, int seq_len, float scale, float eps, int kv_head0, int kv_heads)
{
    const char *what = "attention_prefill_fused_gqa_heads";
    if (!check_heads(kv_head0, kv_heads, what)) return 1;
    return prefill_fused_impl(q_raw, k_raw, v_raw, in_dtype, q_norm, k_norm, token_cos, token_sin, cache, layer_idx,
                              output, out_dtype, seq_len, scale, eps, kv_head0, kv_heads, 1, NULL, NULL, 0, what);
}

int attn_heads_to_tokens(const void *gathered, void *output, int seq_len, int dtype)
{
    const char *what = "attn_heads_to_tokens";
    if (dtype != ATTN_DT_F32 && dtype != ATTN_DT_BF16) {
        tyb_set_error("%s: unknown element type", what);
        return 1;
    }
    if (seq_len < 0 || !gathered || !output) {
        tyb_set_error("%s: bad arguments", what);
        return 1;
    }
    if (seq_len == 0) return 0;
    const int a = tyb_is_device_ptr(gathered), b = tyb_is_device_ptr(output);
    if (a < 0 || b < 0) return 1;
    if (!a || !b) {
        tyb_set_error("%s: gathered and output must be device memory", what);
        return 1;
    }
    if (!tyb_aligned16(gathered, what) || !tyb_aligned16(output, what)) return 1;
    return tyb_cuda_ok(tyb_heads_to_tokens_launch(gathered, output, seq_len, dtype == ATTN_DT_BF16 ? 2 : 4, tyb_stream()),
                       what)
               ? 0
               : 1;
}

int tyb_prefill_sharded(const void *q_raw, const void *k_raw, const void *v_raw, int in_dtype, const float *q_norm,
                        const float *k_norm, const float *token_cos, const float *token_sin, KVCache *cache,
                        int layer_idx, void *own_slot, int seq_len, float scale, float eps, int kv_head0, int kv_heads,
                        const void *xchg_dev, const void *xchg_maps, unsigned int epoch, const char *what)
{
    return prefill_fused_impl(q_raw, k_raw, v_raw, in_dtype, q_norm, k_norm, token_cos, token_sin, cache, layer_idx,
                              own_slot, ATTN_DT_BF16, seq_len, scale, eps, kv_head0, kv_heads, 0,
                              (const tyb_prefill_x *)xchg_dev, xchg_maps, epoch, what);
}
