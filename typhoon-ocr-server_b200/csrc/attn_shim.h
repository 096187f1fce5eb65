/*
 * attn_shim.h -- the thin C interface between the host C of this library
 * (attention.c, kv_cache.c, scratch.c) and its sm_100a kernels (*.cu).
 *
 * Every launcher takes DEVICE pointers only, enqueues on `stream` (a
 * cudaStream_t; NULL = the legacy default stream) and returns a cudaError_t
 * value (0 = success).  Nothing here synchronises; the host C decides when the
 * caller's contract needs a synchronous return.
 */
#ifndef TYB_ATTN_SHIM_H
#define TYB_ATTN_SHIM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element type of KV-cache rows and of staged activations. */
enum { TYB_F32 = 0, TYB_BF16 = 1 };

/* Bits of the device status word (tyb_status_fetch). */
#define TYB_STATUS_WAIT_TIMEOUT 0x1u /* an mbarrier wait ran past its time limit */
#define TYB_STATUS_BAD_ARGUMENT 0x2u /* a kernel found an index outside its buffers */

/* One sequence's K and V rows for ONE layer, head-first:
 * element (kv_head h, row r, dim d) at base + ((size_t)h * row_capacity + r) * 128 + d. */
typedef struct {
    const void *k;
    const void *v;
    int kv_len;       /* rows attended: [0, kv_len) */
    int row_capacity; /* rows allocated per head (the cache's max_seq_len) */
    /* Single-sequence launches only (NULL otherwise): the same-shaped rows of the layer the
     * next call will read.  The FP32-cache kernel asks L2 for its split's row range there once
     * its tiles are requested, so the next layer's launch finds its rows in L2 (a hint: no data
     * dependence). */
    const void *pf_k;
    const void *pf_v;
} tyb_seq_kv;

/* ---- split-KV flash decoding (decode.cu) ------------------------------------------ */

/* Rows per split and split count the decode kernel will use for a batch whose
 * longest sequence has max_kv_len rows. */
void tyb_decode_plan(int batch, int max_kv_len, int kv_dtype, int *chunk_rows, int *nsplit);

/* Floats of split workspace and counters needed for tyb_decode_launch. */
size_t tyb_decode_partial_floats(int batch, int nsplit);

/* q, out: [batch][16][128] fp32.  seqs_dev: device array of `batch` descriptors, or
 * NULL with batch == 1 to use `one`.  partials: >= tyb_decode_partial_floats floats;
 * counters: batch*8 zeroed words (the kernel leaves them zeroed). */
int tyb_decode_launch(const float *q, float *out, const tyb_seq_kv *seqs_dev, tyb_seq_kv one,
                      int batch, int max_kv_len, int kv_dtype, float scale, float *partials,
                      unsigned int *counters, void *stream);

/* tyb_decode_launch plus the fused KV append and early streaming:
 * k_new/v_new: NULL, or [batch][8][128] fp32 rows that are written at row kv_len-1 of each
 * sequence's cache and attended to.
 * prefetch_rows: cache rows [0, prefetch_rows) may be read before the kernel waits for the
 * previous kernel in the stream (single-sequence form only; rows the previous launch
 * wrote must lie at or above it). */
int tyb_decode_launch_ex(const float *q, float *out, const tyb_seq_kv *seqs_dev, tyb_seq_kv one,
                         int batch, int max_kv_len, int kv_dtype, float scale, float *partials,
                         unsigned int *counters, const float *k_new, const float *v_new, int prefetch_rows,
                         void *stream);
/* tyb_decode_launch_ex for KV heads [kvh0, kvh0 + nkvh) only; `out` points at the row of query
 * head 2 kvh0 (the shard's rows [2 nkvh][128] are contiguous). */
/* inl: NULL, or for one sequence (no gather, no QK prep) host memory passed as the launch's own
 * parameters: a copy of q [16][128], the kernel reading q from there (q is not dereferenced);
 * with TYB_DEC_INLINE_ROW in flags, a page-locked slot [K row 1024][V row 1024][q 2048] floats,
 * the kernel reading q and the appended row from there (q / k_new / v_new not dereferenced). */
int tyb_decode_launch_heads(const float *q, float *out, const tyb_seq_kv *seqs_dev, tyb_seq_kv one, int batch,
                            int max_kv_len, int kv_dtype, float scale, float *partials, unsigned int *counters,
                            const float *k_new, const float *v_new, int prefetch_rows, int kvh0, int nkvh,
                            int flags, const void *gather, const float *inl, void *stream);
/* QK-RMSNorm (q_norm / k_norm, eps) and rotate_half M-RoPE with one token's cos / sin [64],
 * applied by the decode kernels on load: all device memory. */
typedef struct {
    const float *q_norm, *k_norm, *cos, *sin;
    float eps;
} tyb_qk_prep;
/* tyb_decode_launch_ex for one sequence with a BF16 cache, all 8 KV heads, device q/k/v, the raw
 * query q_raw [16][128] and raw key row k_raw [8][128] normed and rotated by `prep` on load (the
 * cache receives the normed, rotated K row and v_new as given). */
int tyb_decode_launch_fused(const float *q_raw, float *out, tyb_seq_kv one, int kv_len, float scale, float *partials,
                            unsigned int *counters, const float *k_raw, const float *v_new, int prefetch_rows,
                            const tyb_qk_prep *prep, void *stream);
/* Decode output gather over NVLink (decode.cu): this rank's exchange buffer and peers'. */
int tyb_gather_init(int rank, int world);
int tyb_gather_handle(void *handle_out);            /* 64-byte cudaIpcMemHandle_t */
int tyb_gather_connect(const void *handles);         /* world x 64 bytes, rank order */
const void *tyb_gather_dev(int *world, int *rank);   /* NULL until connected */
void tyb_gather_close(void);
/* Encodes into `map` (a CUtensorMap: 128 bytes, 64-byte aligned) rows [0, rows) of the 8
 * heads of one layer's BF16 cache slab (head stride row_capacity rows) as a 3-D tensor
 * {128 dims, rows, 8 heads}, copied in 128-byte-swizzled boxes of {64, box_rows, 1}; rows
 * past `rows` read as zeros.  0 on success. */
int tyb_encode_rows_map(void *map, const void *base, int rows, int row_capacity, int box_rows);
/* Bytes of the tensor maps tyb_decode_launch_batched uploads for `batch` sequences. */
size_t tyb_decode_maps_bytes(int batch);
/* Decode for a request batch over BF16 caches on the tensor-core kernel: uploads, in one copy
 * into `upload` (device, 64-byte aligned, tyb_decode_maps_bytes(batch) + batch descriptors),
 * two tensor maps per sequence followed by the descriptors `seqs_host`, then launches.  q and
 * out are device [batch][16][128]; partials/counters as for tyb_decode_launch. */
int tyb_decode_launch_batched(const float *q, float *out, const tyb_seq_kv *seqs_host, void *upload, int batch,
                              int max_kv_len, float scale, float *partials, unsigned int *counters, void *stream);
/* flags of tyb_decode_launch_heads: q, k_new and v_new are device memory (not page-locked host
 * memory mapped into the device), so their L2 lines may be requested before the dependency wait. */
#define TYB_DEC_DEVICE_SMALL 1
/* flags: `counters` holds TYB_DEC_WIDE_COUNTER_WORDS zeroed words (8 head counters, then 32 group
 * counters per KV head), so one sequence split over more than 32 CTAs per head is merged in two
 * levels (groups of 16 records in parallel, then the group records). */
#define TYB_DEC_WIDE_COUNTERS 2
#define TYB_DEC_WIDE_COUNTER_WORDS (8 + 8 * 32)
/* flags: `inl` is the whole slot [K row][V row][q] (see tyb_decode_launch_heads). */
#define TYB_DEC_INLINE_ROW 4
/* Relayout of a gathered head-major tensor [16][S][128] into token-major [S][16][128]
 * (elem_bytes 2 or 4). */
int tyb_heads_to_tokens_launch(const void *src, void *dst, int S, int elem_bytes, void *stream);

/* ---- tensor-core prefill (prefill_tc.cu) ---------------------------------------------- */

/* Prefill output exchange of KV-head sharding (shard.c): every rank's buffer is a header of
 * TYB_PX_HEADER_BYTES (flags[8]: the last call whose output rank r has stored here; then the
 * rank's count of finished work items of the current call) followed by two token-major
 * [max_tokens][16][128] BF16 slots, used by call parity.  The device table lists the buffers of
 * all ranks (peers' through CUDA IPC). */
#define TYB_PX_HEADER_BYTES 256
typedef struct {
    void *base[8];
    int rank;
    int world;
    long long slot_elems; /* max_tokens * 16 * 128 */
} tyb_prefill_x;

/* Raw K/V rows [S][8][128] (fp32, or bf16 when in_bf16) -> BF16 cache rows [pos0, pos0+S) of
 * one layer (layout of tyb_seq_kv): K through RMSNorm(k_norm) and rotate_half M-RoPE with the
 * per-token cos/sin [S][64]; V as is.  KV heads [kvh0, kvh0 + nkvh) only.  A programmatic
 * dependent of the previous kernel in the stream (it waits for it before reading anything). */
int tyb_kv_prep_launch(const void *k_raw, const void *v_raw, int in_bf16, const float *k_norm, const float *cos,
                       const float *sin, void *k_dst, void *v_dst, int row_capacity, int pos0, int S, float eps,
                       int kvh0, int nkvh, void *stream);

/* Causal attention of Sq raw queries [Sq][16][128] (fp32 or bf16; RMSNorm(q_norm) + M-RoPE
 * applied on load) over BF16 cache rows [0, pos_offset + Sq) of one layer; query i sits at
 * position pos_offset + i.  KV heads [kvh0, kvh0 + nkvh) and their query heads only.
 * Output [Sq][16][128], or with out_head_major the shard [2 nkvh][Sq][128]; fp32 or bf16.
 * Launched as a programmatic dependent of the previous kernel in the stream, which must be the
 * tyb_kv_prep_launch of the same rows (it starts before that kernel completes; its TMA producer
 * waits for it before reading the cache, and then lets the next kernel in the stream launch).
 * xchg_dev (device table, or NULL): the output rows go, token-major BF16, into slot (epoch & 1)
 * of EVERY rank's exchange buffer instead of `out` (TMA stores through xchg_maps, tyb_prefill_x_maps),
 * and the kernel returns only once all ranks' rows of call `epoch` are in this rank's buffer
 * (bounded wait). */
int tyb_prefill_tc_launch(const void *q, int q_bf16, const float *q_norm, const float *cos, const float *sin,
                          const void *k_cache, const void *v_cache, int row_capacity, void *out, int out_bf16,
                          int Sq, int pos_offset, float scale, float eps, int kvh0, int nkvh, int out_head_major,
                          const tyb_prefill_x *xchg_dev, const void *xchg_maps, unsigned int epoch, void *stream);
/* The TMA tensor maps the sharded prefill stores its output tiles through (xchg_maps of
 * tyb_prefill_tc_launch): one per rank over the two slots of that rank's exchange buffer
 * (bases[p]: the buffer, as tyb_prefill_x.base), written to maps_out (8 x 128 bytes, 64-byte
 * aligned).  0 on success. */
#define TYB_PX_MAPS_BYTES (8 * 128)
int tyb_prefill_x_maps(void *const *bases, int world, int max_tokens, void *maps_out);

/* ---- tensor-core prefill at the FP32 bar (prefill_tc32.cu) ----------------------------- */

/* FP32 K and V rows [0, n) of the 8 KV heads, element (row r, head h, dim d) at
 * base + r*row_stride + h*head_stride + d, split into head-first [8][n][128] BF16 pairs:
 * hi = bf16(x), lo = bf16(x - hi). */
int tyb_kv_split_launch(const float *k, const float *v, long long row_stride, long long head_stride, int n,
                        void *k_hi, void *k_lo, void *v_hi, void *v_lo, void *stream);
/* As tyb_kv_split_launch, with the n rows going to rows [row0, row0 + n) of [8][cap][128] arrays
 * (the chunks of a pipelined split). */
int tyb_kv_split_rows_launch(const float *k, const float *v, long long row_stride, long long head_stride, int n,
                             int row0, int cap, void *k_hi, void *k_lo, void *v_hi, void *v_lo, void *stream);

/* Causal attention of Sq queries q [Sq][16][128] fp32 (already normalised and rotated) into
 * out [Sq][16][128] fp32: query i sees keys k <= pos_offset + i with k < total_kv (>= 1).  K and
 * V as head-first [8][head_rows][128] BF16: hi / lo pairs from tyb_kv_split_launch (FP32-accurate
 * products, three BF16 MMAs each), or the rows of a BF16 cache with k_lo = v_lo = NULL.
 * Launched as a programmatic dependent of the previous kernel in the stream (it waits for that
 * kernel before reading anything). */
int tyb_prefill_tc32_launch(const float *q, float *out, int Sq, int pos_offset, int total_kv, const void *k_hi,
                            const void *k_lo, const void *v_hi, const void *v_lo, int head_rows, float scale,
                            void *stream);

/* ---- KV-cache row writes (kv_write.cu) -------------------------------------------- */

/* Token-major fp32 rows [S][8][128] -> head-first cache rows [pos0, pos0+S) of one layer
 * (layout of tyb_seq_kv), converting to the cache's element type. */
int tyb_kv_scatter_launch(const float *k_src, const float *v_src, void *k_dst, void *v_dst,
                          int row_capacity, int pos0, int S, int kv_dtype, void *stream);

/* ---- status word -------------------------------------------------------------------- */

/* Limit of the kernels' bounded waits on the current device (default 2 s): kernels launched
 * afterwards give up after `ns` nanoseconds and raise TYB_STATUS_WAIT_TIMEOUT. */
int tyb_set_wait_limit(unsigned long long ns);
unsigned long long tyb_wait_limit(void);

/* Copy the status word to *bits after all work on `stream`, then clear it. */
int tyb_status_fetch(unsigned int *bits, void *stream);
/* Device address of the status word on the current device (NULL on failure). */
unsigned int *tyb_status_word(void);
/* Status mirror (a page-locked host word that kernels flag when they raise a status bit):
 * set up for the current device (0 or a cudaError_t); its host view, or NULL when the
 * current device has none; its device view, or NULL. */
int tyb_status_mirror_setup(void);
unsigned int *tyb_status_mirror_host(void);
unsigned int *tyb_status_mirror_device(void);

#ifdef __cplusplus
}
#endif
#endif
