/*
 * host_internal.h -- shared declarations of the host C layer (runtime.c, kv_cache.c,
 * scratch.c, attention.c).  Not part of the public interface.
 */
#ifndef TYB_HOST_INTERNAL_H
#define TYB_HOST_INTERNAL_H

#include <stddef.h>
#include <stdint.h>

#include "attn_shim.h"
#include "kv_cache.h"

#ifdef __cplusplus
extern "C" {
#endif

#define TYB_CACHE_MAGIC 0x54594243u /* "TYBC" */
#define TYB_ROW_FLOATS (KV_NUM_KV_HEADS * KV_HEAD_DIM) /* 1024: one token of K or V */
#define TYB_Q_FLOATS (16 * KV_HEAD_DIM)               /* 2048: one token of Q / output */
/* Longest cache accepted (sizes the per-cache decode split workspace). */
#define TYB_MAX_SEQ 262144

/* Device cache.  `pub` is the first member, so the KVCache* handed to callers converts
 * back to this struct; callers only ever touch pub's fields. */
typedef struct {
    KVCache pub;
    uint32_t magic;
    int dtype;               /* TYB_F32 / TYB_BF16 */
    int device;              /* CUDA device current at allocation */
    size_t elem_bytes;       /* 4 or 2 */
    void *k_slab, *v_slab;   /* [28][8][max_seq][128] elements */
    float *d_out;            /* [16][128] staging of a host output (decode) */
    float *d_kv_stage;       /* [2][max_seq][8][128] fp32 staging of host K/V rows (>= 16 KB); also the
                              * device copy of a decode call's host inputs (one slot) */
    float *d_partials;       /* split-KV workspace of the decode kernel */
    unsigned int *d_counters;/* split tickets: 8 per head, then 32 group counters per head (TYB_DEC_WIDE_COUNTER_WORDS), kept zero between launches */
    /* Deferred single-row appends from host memory (kv_cache_append as kernel/decoder.c:96-100
     * calls it): the row is copied here at once, and written to the cache by the next launch that
     * touches its layer -- normally the attention_decode_gqa of the same step, which then appends
     * and attends in one kernel. */
    float *h_rows;           /* page-locked, device-mapped [28][4][1024]: per layer the staged K row, V
                              * row, then room for a host query [16][128] copied beside them (the
                              * parameter block of a decode launch from host inputs) */
    float *h_rows_dev;       /* its device view */
    void *row_ev[KV_NUM_LAYERS]; /* cudaEvent_t: recorded after the launch that read the layer's slot */
    unsigned char slot_read[KV_NUM_LAYERS]; /* row_ev recorded since the host last waited for it */
    int pending[KV_NUM_LAYERS];  /* row the layer's staged row goes to, or -1 */
    /* In the same page-locked block, after the slots: the [16][128] output staging of a pageable
     * host output (written by the decode kernel through its device view, copied out after the
     * call's wait). */
    float *h_out, *h_out_dev;
} tyb_cache;

/* Writes (cache, layer)'s deferred row, if any, on the calling thread's stream; every path that
 * reads or writes the layer's rows calls it first.  1 on success, else 0 with the error set. */
int tyb_flush_pending(tyb_cache *t, int layer, const char *what);
/* The layer's staging slot: K row [8][128], V row [8][128], query [16][128] (4096 floats). */
#define TYB_SLOT_FLOATS (4 * TYB_ROW_FLOATS)
/* The page-locked block: the 28 slots, then the output staging. */
#define TYB_PINNED_FLOATS ((size_t)KV_NUM_LAYERS * TYB_SLOT_FLOATS + TYB_Q_FLOATS)
/* Host output of a blocking decode call, stored by the kernel through a device mapping: filled
 * with TYB_UNWRITTEN before the launch (tyb_mark_unwritten), then tyb_wait_output waits until no
 * word holds it (or for the stream when a status bit is raised or the stream goes idle first);
 * 1 on success, else 0 with the error set. */
#define TYB_UNWRITTEN 0xFFFFFFFFu
void tyb_mark_unwritten(float *out, size_t n);
int tyb_wait_output(const float *out, size_t n, void *stream, const char *what);
static inline float *tyb_row_slot(const tyb_cache *t, int layer) { return t->h_rows + (size_t)layer * TYB_SLOT_FLOATS; }
/* The slots (page-locked, device-mapped) and their events, set up on first use; 1 on success. */
int tyb_slots_ready(tyb_cache *t, const char *what);
/* Records the layer's "slot consumed" event after a launch that read the slot. */
int tyb_slot_consumed(tyb_cache *t, int layer, void *stream, const char *what);
/* Before the host rewrites the layer's slot: waits for the last launch that read it, if one has
 * since the last wait (a launch that takes the slot as its parameter block copies it at the
 * launch and records nothing).  1 on success. */
int tyb_slot_wait(tyb_cache *t, int layer, const char *what);

/* The cache behind a KVCache*, or NULL (error set) if this library did not make it. */
tyb_cache *tyb_cache_from(const KVCache *c);

/* Device address of row 0 of (layer, head) in a slab. */
static inline void *tyb_slab_head(const tyb_cache *c, void *slab, int layer, int head)
{
    size_t rows = (size_t)c->pub.max_seq_len;
    return (char *)slab + (((size_t)layer * KV_NUM_KV_HEADS + head) * rows) * KV_HEAD_DIM * c->elem_bytes;
}

/* K/V rows of (cache, layer) for a single-sequence decode launch attending kv_len rows.  pf_k /
 * pf_v point at the rows the next decode call of kernel/decoder.c's layer loop reads: layer + 1,
 * and layer 0 (the next step) after the last layer.  Rows below seq_len there are final before
 * the step starts, so the launch asks L2 for them while it runs. */
static inline tyb_seq_kv tyb_layer_rows(const tyb_cache *c, int layer, int kv_len)
{
    const int next = layer + 1 < KV_NUM_LAYERS ? layer + 1 : 0;
    tyb_seq_kv s;
    s.k = tyb_slab_head(c, c->k_slab, layer, 0);
    s.v = tyb_slab_head(c, c->v_slab, layer, 0);
    s.kv_len = kv_len;
    s.row_capacity = c->pub.max_seq_len;
    s.pf_k = tyb_slab_head(c, c->k_slab, next, 0);
    s.pf_v = tyb_slab_head(c, c->v_slab, next, 0);
    return s;
}

/* Errors: thread-local message, "" when none. */
void tyb_set_error(const char *fmt, ...);

/* 1 when p is 16-byte aligned (the kernels read and write rows with 16-byte vector accesses);
 * otherwise 0 with the error set, so a misaligned buffer is refused before any launch. */
static inline int tyb_aligned16(const void *p, const char *what)
{
    if (((uintptr_t)p & 15u) == 0) return 1;
    tyb_set_error("%s: buffer %p is not 16-byte aligned", what, p);
    return 0;
}

/* 1 when err == 0 (cudaSuccess); otherwise records "<what>: <cuda error string>", returns 0. */
int tyb_cuda_ok(int err, const char *what);

/* The calling thread's stream (NULL = legacy default stream). */
void *tyb_stream(void);

/* 1 when p is device (or managed) memory usable by kernels, 0 when host memory,
 * -1 on error (error set). */
int tyb_is_device_ptr(const void *p);

/* Where p lives, for the calls that take host or device buffers:
 *   TYB_MEM_DEVICE  device or managed memory: *view = p
 *   TYB_MEM_PINNED  page-locked host memory mapped into the device's address space: *view is
 *                   the device-side address (kernels read and write it over the bus)
 *   TYB_MEM_HOST    pageable host memory: *view = NULL, the data must be copied
 * Returns -1 on error (error set). */
enum { TYB_MEM_HOST = 0, TYB_MEM_DEVICE = 1, TYB_MEM_PINNED = 2 };
int tyb_residency(const void *p, void **view);

/* cudaMalloc / cudaHostAlloc that honour the TYB_FAULT_ALLOC failure injection (runtime.c);
 * 1 on success, else 0 with *p = NULL and the error set. */
int tyb_dev_alloc(void **p, size_t bytes, const char *what);
int tyb_host_alloc(void **p, size_t bytes, unsigned int flags, const char *what);

/* The current device's workspace slots, grown on demand (attn_workspace_reserve sizes them
 * ahead); NULL on failure (error set). */
enum { TYB_WS_Q, TYB_WS_K, TYB_WS_V, TYB_WS_OUT, TYB_WS_PARTIALS, TYB_WS_COUNTERS, TYB_WS_DESC,
       TYB_WS_COUNT };
void *tyb_workspace(int slot, size_t bytes);

/* Device buffers handed out by decoder_scratch_alloc, so attention_prefill_gqa can tell
 * whether a q_hm/k_hm/v_hm/o_hm pointer is ours and how large it is. */
void   tyb_registry_add(const void *p, size_t bytes);
void   tyb_registry_remove(const void *p);
size_t tyb_registry_size(const void *p); /* 0 when unknown */

/* Which cache rows the most recent launch of this thread wrote.  A kernel may read rows
 * before waiting on its predecessor (programmatic dependent launch) only if that
 * predecessor did not write them: every launch of this library waits on its own
 * predecessor before it lets the next one start, so writes two or more launches back
 * are complete.
 *   tyb_note_write: the launch just queued wrote rows >= lo of (cache, layer).
 *   tyb_note_nowrite: the launch just queued wrote no cache rows.
 *   tyb_prefetch_rows: how many leading rows of (cache, layer) the next launch may read
 *                      early (at most `rows`). */
void tyb_note_write(const void *cache, int layer, int lo, void *stream);
void tyb_note_nowrite(void *stream);
int  tyb_prefetch_rows(const void *cache, int layer, int rows);

/* The fused prefill of attention_prefill_fused_gqa_heads in its sharded form: output rows into
 * every rank's exchange slot (xchg_dev: the device tyb_prefill_x of shard.c, xchg_maps its
 * tyb_prefill_x_maps; own_slot: this rank's slot of call `epoch`, for the argument checks).
 * 0 on success. */
int tyb_prefill_sharded(const void *q_raw, const void *k_raw, const void *v_raw, int in_dtype, const float *q_norm,
                        const float *k_norm, const float *token_cos, const float *token_sin, KVCache *cache,
                        int layer_idx, void *own_slot, int seq_len, float scale, float eps, int kv_head0, int kv_heads,
                        const void *xchg_dev, const void *xchg_maps, unsigned int epoch, const char *what);

/* Wait for `stream`, then check the device status word.  1 when all is well;
 * otherwise 0 with the error set. */
int tyb_finish(void *stream, const char *what);

#ifdef __cplusplus
}
#endif
#endif
