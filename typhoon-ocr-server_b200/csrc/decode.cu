// decode.cu -- split-KV flash decoding for one new token per sequence, optionally fused
// with the KV append of that token.
//
// Replaces the reference's per-KV-head CPU worker (kernel/attention.c:158-204: for each
// KV head and its two query heads, scores = q.K*scale over kv_len rows, max, exp, sum,
// normalise, out = sum p*V) and, fused, kernel/kv_cache.c:53-65 (the new row written at
// row seq_len first).  One CTA owns one (sequence, KV head, split of rows):
//   1. the split's K and V rows are requested into shared memory by TMA on two mbarriers.
//      Kernels are launched with programmatic dependent launch, so the next kernel's CTAs are
//      resident early and request their rows BEFORE griddepcontrol.wait (only rows the host
//      knows the previous launch did not write).  On B200 the completion of such copies is
//      held until the previous grid has finished, but their data moves meanwhile: at 4K the
//      K tile lands ~0.5 us after the wait returns, against ~2.6 us of HBM time for a layer;
//   2. after the wait: the query (and the new row, written to the cache and into its
//      slot), scores of both query heads, max and exp2 per head;
//   3. p.V for both heads from the same V bytes (GQA pair read once);
//   4. the split's (max, sum, unnormalised o) goes to a workspace record; the CTA that
//      takes the last ticket merges all records (up to 32 with plain L2 loads, 33-64 pulled
//      into shared memory by bulk copies, more in two levels of groups) and writes the
//      output.  No second launch.
// Three kernels implement it: decode_mma_kernel (one sequence whose splits fit one wave, BF16
// cache: the contractions on the tensor cores through mma.sync, tiles by TMA tensor copies),
// decode_stream_kernel (longer sequences and request batches, BF16: each CTA streams a span of
// rows in double-buffered stages with an online softmax) and decode_split_kernel<T> (FP32
// caches: CUDA-core dot products, tiles by 1-D bulk copies).
// Bandwidth-bound: 2 * kv_len * 128 * sizeof(T) bytes per (sequence, KV head).
#include <cuda.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "host_internal.h"

namespace tyb {

constexpr int kDecThreads = 256;
constexpr int kRowGroups = kDecThreads / 16;  // p.V row groups (16 lanes per row)
constexpr int kRec = 4 + 2 * kD;              // record: m0 l0 m1 l1 | o0[128] | o1[128]
// p.V reduction area: [16 row groups][2 heads][128] partial outputs + [16][2] partial sums.
constexpr int kRedBytes = (kRowGroups * 2 * kD + kRowGroups * 2) * (int)sizeof(float);

template <typename T>
struct DecodeTile {
    // Rows per split: bounded so K+V of two CTAs fit in one SM's shared memory.
    static constexpr int kMaxChunk = sizeof(T) == 2 ? 192 : 96;
};

struct DecodeArgs {
    const float* q;
    float* out;
    const tyb_seq_kv* seqs;
    tyb_seq_kv one;
    const float* k_new;  // [batch][8][128] fp32 rows appended at row kv_len-1, or NULL
    const float* v_new;
    float scale_log2;
    int chunk;
    int nsplit_max;
    int prefetch_rows;  // rows [0, prefetch_rows) may be requested before the dependency wait
    float* partials;
    unsigned int* counters;
    int kvh0;  // KV heads [kvh0, kvh0 + gridDim.y); out points at query head 2 kvh0's row
    int prefetch_small;  // q, k_new, v_new are device memory: ask L2 for their lines early
};

// Inputs of a call whose inputs are host memory, carried in the launch's own parameters (kernel
// parameter space holds up to 32 KB): they reach the GPU with the launch itself, so no copy is
// queued ahead of the kernel.  Read through the parameter's address (hence __grid_constant__;
// 16-byte aligned for the vector loads).  Two forms:
//   DecodeInline     the query [16][128] only, for a call that blocks on a host output: the
//                    appended K/V row, read by one CTA per KV head only, comes through the
//                    device mapping of the page-locked slot it is staged in (k_new / v_new) --
//                    0.6 us less per blocking call than a 16 KB block (the launch copies and
//                    uploads half the bytes), and the output is written after the row is read,
//                    so the slot is free when the call returns;
//   DecodeInlineRow  the slot's whole contents, K row, V row, query (16 KB), for a call that
//                    returns before its kernel has run (a device output): nothing on the device
//                    reads the slot, so the host may rewrite it at once (with the row read
//                    through the mapping, the slot's next writer had to wait for the launch:
//                    10.2 against 7.1 us per call back to back).
struct __align__(16) DecodeInline {
    float q[kHq * kD];
};
struct __align__(16) DecodeInlineRow {
    float k[kHkv * kD];
    float v[kHkv * kD];
    float q[kHq * kD];
};
struct DecodeNoInline {  // the inputs are device memory, read through the argument pointers
    int unused;
};
template <typename In>
constexpr bool kIsInline = !std::is_same<In, DecodeNoInline>::value;

// The query / new-row sources of a launch: the argument pointers, or the parameter copies (k and
// v only in DecodeInlineRow, and when the call appends a row: the argument pointers then only say
// whether it does).
__device__ __forceinline__ void inline_inputs(const DecodeNoInline&, const float*&, const float*&, const float*&) {}
__device__ __forceinline__ void inline_inputs(const DecodeInline& in, const float*& q, const float*&, const float*&)
{
    q = in.q;
}
__device__ __forceinline__ void inline_inputs(const DecodeInlineRow& in, const float*& q, const float*& k,
                                              const float*& v)
{
    q = in.q;
    if (k) k = in.k;
    if (v) v = in.v;
}


__device__ __forceinline__ float fast_exp2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename T>
__host__ __device__ constexpr size_t dec_kv_bytes(int chunk)
{
    return (size_t)chunk * kD * sizeof(T);
}

// Shared memory: [K (>= kRedBytes, reused for the p.V reduction and merge headers)]
// [V (reused for merge weights)] [scores 2 x chunk] [stat 24] [3 mbarriers] [flag].
template <typename T>
__host__ __device__ constexpr size_t dec_k_region(int chunk)
{
    return dec_kv_bytes<T>(chunk) > (size_t)kRedBytes ? dec_kv_bytes<T>(chunk) : (size_t)kRedBytes;
}

template <typename T>
__host__ __device__ constexpr size_t decode_smem_bytes(int chunk)
{
    return dec_k_region<T>(chunk) + dec_kv_bytes<T>(chunk) + sizeof(float) * (2 * chunk + 24) + 3 * sizeof(uint64_t) +
           16;
}

// The 16 dims of a 128-dim row that lane part p (0..7) of an 8-lane row group takes in the
// score pass, chosen so that the 8 lanes of a row read 8 different 16-byte units of a
// 128-byte line at every load (no bank conflicts across the 4 rows of a warp pass): BF16 rows
// (256 B) in two 8-dim chunks [8p, 8p+8) and [64+8p, 64+8p+8); FP32 rows (512 B) in four
// 4-dim chunks [32c+4p, 32c+4p+4).  The query uses the same dims.
__device__ __forceinline__ void load_lane16(const __nv_bfloat16* row, int p, float (&x)[16])
{
    load8(row + 8 * p, *reinterpret_cast<float(*)[8]>(&x[0]));
    load8(row + 64 + 8 * p, *reinterpret_cast<float(*)[8]>(&x[8]));
}

__device__ __forceinline__ void load_lane16(const float* row, int p, float (&x)[16])
{
#pragma unroll
    for (int c = 0; c < 4; c++) {
        const float4 v = *reinterpret_cast<const float4*>(row + 32 * c + 4 * p);
        x[4 * c] = v.x;
        x[4 * c + 1] = v.y;
        x[4 * c + 2] = v.z;
        x[4 * c + 3] = v.w;
    }
}

template <typename T>
__device__ __forceinline__ void load_query16(const float* q, int p, float (&x)[16])
{
    if (sizeof(T) == 2) {
        load8(q + 8 * p, *reinterpret_cast<float(*)[8]>(&x[0]));
        load8(q + 64 + 8 * p, *reinterpret_cast<float(*)[8]>(&x[8]));
    } else {
        load_lane16(q, p, x);
    }
}

// Merge of the `nsplit` split records of one (sequence, KV head) by the CTA that took the last
// ticket; every thread of the CTA calls it.  Records arrive in shared memory (`region`, the
// CTA's free K/V space) in batches by one bulk copy each on `bar` (phase 0 first); every
// thread then merges one output element (h, d) = (tid / 128, tid % 128), with an online
// maximum across batches, and writes out[h * 128 + d].  red32: 32 floats of scratch.
// False when a wait ran out (the status word is raised).
__device__ __forceinline__ bool merge_records(const float* recs, int nsplit, float* region, size_t region_bytes, uint64_t* bar,
                              float* red32, float* out)
{
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int h = tid >> 7;
    const int d = tid & 127;
    const int cap = (int)(region_bytes / (sizeof(float) * (kRec + 2)));
    float* wts = region + (size_t)cap * kRec;  // [cap][2]
    float run0 = -INFINITY, run1 = -INFINITY;  // running max of each head (uniform)
    float L = 0.f, O = 0.f;                     // this thread's head h, element d
    uint32_t phase = 0;
    for (int j0 = 0; j0 < nsplit; j0 += cap) {
        const int nb = min(cap, nsplit - j0);
        __syncthreads();  // the previous batch is consumed
        if (tid == 0) {
            fence_proxy_async_smem();  // the region's earlier (generic) reads come before the copy's writes
            const uint32_t bytes = (uint32_t)nb * kRec * sizeof(float);
            mbar_arrive_expect_tx(bar, bytes);
            bulk_g2s(region, recs + (size_t)j0 * kRec, bytes, bar);
        }
        if (__syncthreads_or(!mbar_wait_bounded(bar, phase, wait_limit_ns(), TYB_STATUS_WAIT_TIMEOUT))) return false;
        phase ^= 1u;
        // Batch maximum of each head: a block reduction over the records' headers.
        float x0 = -INFINITY, x1 = -INFINITY;
        for (int j = tid; j < nb; j += kDecThreads) {
            x0 = fmaxf(x0, region[(size_t)j * kRec + 0]);
            x1 = fmaxf(x1, region[(size_t)j * kRec + 2]);
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
            x0 = fmaxf(x0, __shfl_xor_sync(0xffffffffu, x0, off));
            x1 = fmaxf(x1, __shfl_xor_sync(0xffffffffu, x1, off));
        }
        if (lane == 0) {
            red32[warp] = x0;
            red32[16 + warp] = x1;
        }
        __syncthreads();
        float n0 = run0, n1 = run1;
#pragma unroll
        for (int w = 0; w < kDecThreads / 32; w++) {
            n0 = fmaxf(n0, red32[w]);
            n1 = fmaxf(n1, red32[16 + w]);
        }
        // Weights of this batch's records against the new maxima.
        for (int j = tid; j < nb; j += kDecThreads) {
            wts[2 * j] = fast_exp2(region[(size_t)j * kRec + 0] - n0);
            wts[2 * j + 1] = fast_exp2(region[(size_t)j * kRec + 2] - n1);
        }
        __syncthreads();
        const float alpha = fast_exp2((h ? run1 : run0) - (h ? n1 : n0));  // 0 on the first batch
        L *= alpha;
        O *= alpha;
        const float* lp = region + 1 + 2 * h;
        const float* op = region + 4 + (size_t)h * kD + d;
#pragma unroll 4
        for (int j = 0; j < nb; j++) {
            const float w = wts[2 * j + h];
            L = fmaf(lp[(size_t)j * kRec], w, L);
            O = fmaf(op[(size_t)j * kRec], w, O);
        }
        run0 = n0;
        run1 = n1;
    }
    out[(size_t)h * kD + d] = O / L;
    return true;
}

template <typename T, typename In>
__global__ void __launch_bounds__(kDecThreads, 2) decode_split_kernel(const DecodeArgs a, const __grid_constant__ In in)
{
    extern __shared__ __align__(128) unsigned char smem[];
    const int s = blockIdx.x;
    const int kvh = a.kvh0 + blockIdx.y;
    const int b = blockIdx.z;
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;

    unsigned char* kreg = smem;
    unsigned char* vreg = smem + dec_k_region<T>(a.chunk);
    T* Ks = reinterpret_cast<T*>(kreg);
    T* Vs = reinterpret_cast<T*>(vreg);
    float* sc = reinterpret_cast<float*>(vreg + dec_kv_bytes<T>(a.chunk));  // [2][chunk]
    float* stat = sc + 2 * a.chunk;  // m0 m1 l0 l1, then [8 warps][2] score maxima
    uint64_t* bars = reinterpret_cast<uint64_t*>(stat + 24);  // K rows, V rows, merge records
    int* last_flag = reinterpret_cast<int*>(bars + 3);
    float* red = reinterpret_cast<float*>(kreg);  // [16][2][128], after the scores
    const float* q_src = a.q;
    const float* k_src = a.k_new;
    const float* v_src = a.v_new;
    inline_inputs(in, q_src, k_src, v_src);

    // Split geometry.  The new token's row (fused append) never comes from the cache.
    int kv_len = 0, nsplit = 0, r0 = 0, nrows = 0, tma_rows = 0;
    const T* kh = nullptr;
    const T* vh = nullptr;
    auto geometry = [&](const tyb_seq_kv& seq) {
        kv_len = seq.kv_len;
        nsplit = (kv_len + a.chunk - 1) / a.chunk;
        r0 = s * a.chunk;
        nrows = max(0, min(a.chunk, kv_len - r0));
        tma_rows = max(0, min(nrows, (a.k_new ? kv_len - 1 : kv_len) - r0));
        kh = static_cast<const T*>(seq.k) + (size_t)kvh * seq.row_capacity * kD;
        vh = static_cast<const T*>(seq.v) + (size_t)kvh * seq.row_capacity * kD;
    };
    auto issue = [&]() {
        const uint32_t bytes = (uint32_t)tma_rows * kD * sizeof(T);
        if (bytes) {
            mbar_arrive_expect_tx(&bars[0], bytes);
            bulk_g2s(Ks, kh + (size_t)r0 * kD, bytes, &bars[0]);
            mbar_arrive_expect_tx(&bars[1], bytes);
            bulk_g2s(Vs, vh + (size_t)r0 * kD, bytes, &bars[1]);
        } else {
            mbar_arrive(&bars[0]);
            mbar_arrive(&bars[1]);
        }
    };
    // Single-sequence form: the geometry is in the parameters, so the split's rows are
    // copied before waiting for the previous kernel when that kernel did not write them.
    bool early = false;
    if (!a.seqs) {
        geometry(a.one);
        early = s < nsplit && r0 + tma_rows <= a.prefetch_rows;
    }
    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        mbar_init(&bars[2], 1);
        fence_barrier_init();
        fence_proxy_async_smem();
    }
    __syncthreads();
    // The query and the appended row may be written by the previous kernel, so they are read
    // only after the wait; asking L2 for their lines first is still safe (device writes land in
    // L2, which the later loads read) and takes the DRAM latency off the path after the wait.
    // Plain prefetch instructions, one 128-byte line per lane: q of the two heads (8 lines),
    // then the new K and V rows (4 lines each) in the CTA that appends them.
    if (!kIsInline<In> && a.prefetch_small && warp == 1) {
        const float* line = nullptr;
        if (lane < 8) {
            line = q_src + ((size_t)b * kHq + kGroup * kvh) * kD + lane * 32;
        } else if (lane < 16 && !a.seqs && k_src && kv_len - 1 >= r0 && kv_len - 1 < r0 + nrows) {
            const size_t off = ((size_t)b * kHkv + kvh) * kD + (lane & 3) * 32;
            line = (lane < 12 ? k_src : v_src) + off;
        }
        if (line) asm volatile("prefetch.global.L2 [%0];" ::"l"(line));
    }
    // The next call's rows (tyb_seq_kv.pf_k): asked of L2 right after this split's own copies, so
    // that the next layer's copies hit L2 (at 4K one FP32 layer's K/V is 33.6 MB: it fits in L2
    // beside this one).  Measured at 4K, 28 layers: 362 against 386 us per step.  (The BF16
    // tensor-core form gains nothing from it: its tiles land within ~0.6 us of the dependency
    // release, and the prefetch, issued with the tiles or after the split's work, cost 4-9 %.)
    auto prefetch_next = [&]() {
        if (a.one.pf_k && tma_rows > 0) {
            const size_t off = ((size_t)kvh * a.one.row_capacity + r0) * kD;
            const uint32_t bytes = (uint32_t)tma_rows * kD * sizeof(T);
            bulk_prefetch_l2(static_cast<const T*>(a.one.pf_k) + off, bytes);
            bulk_prefetch_l2(static_cast<const T*>(a.one.pf_v) + off, bytes);
        }
    };
    if (tid == 0 && early) {
        issue();
        prefetch_next();
    }
    // Everything below reads data earlier kernels wrote (descriptors, cache rows, q).
    pdl_wait();
    pdl_trigger();
    if (a.seqs) geometry(a.seqs[b]);
    if (s >= nsplit) return;
    if (tid == 0 && !early) {
        issue();
        if (!a.seqs) prefetch_next();
    }

    // Query vectors of the two heads sharing this KV head, for the scores: 8 lanes per row,
    // lane part p holds the 16 dims of load_lane16.
    const int g16 = lane & 15;
    const int part = lane & 7;
    float q0[16], q1[16];
    {
        const float* qb = q_src + (size_t)b * kHq * kD + (size_t)(kGroup * kvh) * kD;
        load_query16<T>(qb, part, q0);
        load_query16<T>(qb + kD, part, q1);
    }

    // The new token's row (fused append): threads 0..15 write it to the cache and into its
    // slot after the copied rows (K now, V once V has landed).
    const bool has_new = a.k_new && kv_len - 1 >= r0 && kv_len - 1 < r0 + nrows;
    float nk[8], nv[8];
    if (has_new && tid < 16) {
        const size_t off = ((size_t)b * kHkv + kvh) * kD + tid * 8;
        load8(k_src + off, nk);
        load8(v_src + off, nv);
        store8(const_cast<T*>(kh) + (size_t)(kv_len - 1) * kD + tid * 8, nk);
        store8(const_cast<T*>(vh) + (size_t)(kv_len - 1) * kD + tid * 8, nv);
        store8(Ks + (size_t)(kv_len - 1 - r0) * kD + tid * 8, nk);
    }

    // Every thread waits (bounded); the CTA leaves together if any wait ran out.
    if (__syncthreads_or(!mbar_wait_bounded(&bars[0], 0, wait_limit_ns(), TYB_STATUS_WAIT_TIMEOUT))) return;

    // Scores: 8 lanes per row (each 16-byte chunk of a 128-byte line read by one lane: no
    // bank conflicts), 4 rows per warp pass, two passes 32 rows apart interleaved; a 3-level
    // shuffle-xor sum.  Each warp keeps the maximum of its rows per head.
    float* wmax = stat + 4;  // [8 warps][2] -> after the scores, stat[4..] is scratch
    {
        const int rsub = lane >> 3;
        float m0 = -INFINITY, m1 = -INFINITY;
        for (int base = warp * 4; base < nrows; base += 64) {
            const int ra = base + rsub, rb = base + 32 + rsub;
            const int ra_c = min(ra, nrows - 1), rb_c = min(rb, nrows - 1);
            float ka[16], kb[16];
            load_lane16(Ks + (size_t)ra_c * kD, part, ka);
            load_lane16(Ks + (size_t)rb_c * kD, part, kb);
            float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f, a2 = 0.f, a3 = 0.f, b2 = 0.f, b3 = 0.f;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                a0 = fmaf(q0[j], ka[j], a0);
                a1 = fmaf(q1[j], ka[j], a1);
                b0 = fmaf(q0[j], kb[j], b0);
                b1 = fmaf(q1[j], kb[j], b1);
                a2 = fmaf(q0[8 + j], ka[8 + j], a2);
                a3 = fmaf(q1[8 + j], ka[8 + j], a3);
                b2 = fmaf(q0[8 + j], kb[8 + j], b2);
                b3 = fmaf(q1[8 + j], kb[8 + j], b3);
            }
            a0 += a2;
            a1 += a3;
            b0 += b2;
            b1 += b3;
#pragma unroll
            for (int off = 4; off >= 1; off >>= 1) {
                a0 += __shfl_xor_sync(0xffffffffu, a0, off);
                a1 += __shfl_xor_sync(0xffffffffu, a1, off);
                b0 += __shfl_xor_sync(0xffffffffu, b0, off);
                b1 += __shfl_xor_sync(0xffffffffu, b1, off);
            }
            if (part == 0) {
                if (ra < nrows) {
                    const float x0 = a0 * a.scale_log2, x1 = a1 * a.scale_log2;
                    sc[ra] = x0;
                    sc[a.chunk + ra] = x1;
                    m0 = fmaxf(m0, x0);
                    m1 = fmaxf(m1, x1);
                }
                if (rb < nrows) {
                    const float x0 = b0 * a.scale_log2, x1 = b1 * a.scale_log2;
                    sc[rb] = x0;
                    sc[a.chunk + rb] = x1;
                    m0 = fmaxf(m0, x0);
                    m1 = fmaxf(m1, x1);
                }
            }
        }
#pragma unroll
        for (int off = 8; off <= 16; off <<= 1) {
            m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, off));
            m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, off));
        }
        if (lane == 0) {
            wmax[2 * warp] = m0;
            wmax[2 * warp + 1] = m1;
        }
    }
    __syncthreads();

    // exp2 of every score against its head's maximum, all threads at once.
    {
        float M0 = -INFINITY, M1 = -INFINITY;
#pragma unroll
        for (int w = 0; w < kDecThreads / 32; w++) {
            M0 = fmaxf(M0, wmax[2 * w]);
            M1 = fmaxf(M1, wmax[2 * w + 1]);
        }
        for (int i = tid; i < 2 * nrows; i += kDecThreads) {
            const int hh = i >= nrows;
            float* x = sc + hh * a.chunk + (i - hh * nrows);
            *x = fast_exp2(*x - (hh ? M1 : M0));
        }
        __syncthreads();  // every thread has read wmax: stat[0..1] may take the maxima
        if (tid == 0) {
            stat[0] = M0;
            stat[1] = M1;
        }
    }

    if (has_new && tid < 16) store8(Vs + (size_t)(kv_len - 1 - r0) * kD + tid * 8, nv);
    if (__syncthreads_or(!mbar_wait_bounded(&bars[1], 0, wait_limit_ns(), TYB_STATUS_WAIT_TIMEOUT))) return;

    // p.V: thread owns dims [8*g16, +8) of rows rg, rg+16, ...
    const int rg = tid >> 4;
    float o0[8], o1[8];
    float l0 = 0.f, l1 = 0.f;  // this row group's weight sums (used from lane g16 == 0)
#pragma unroll
    for (int j = 0; j < 8; j++) o0[j] = o1[j] = 0.f;
    for (int r = rg; r < nrows; r += kRowGroups) {
        float v8[8];
        load8(Vs + (size_t)r * kD + g16 * 8, v8);
        const float p0 = sc[r], p1 = sc[a.chunk + r];
        l0 += p0;
        l1 += p1;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            o0[j] = fmaf(p0, v8[j], o0[j]);
            o1[j] = fmaf(p1, v8[j], o1[j]);
        }
    }
    store8(red + ((size_t)rg * 2 + 0) * kD + g16 * 8, o0);  // K region is free now
    store8(red + ((size_t)rg * 2 + 1) * kD + g16 * 8, o1);
    float* lred = red + kRowGroups * 2 * kD;  // [16][2]
    if (g16 == 0) {
        lred[2 * rg] = l0;
        lred[2 * rg + 1] = l1;
    }
    __syncthreads();
    if (tid == 0) {
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int g = 0; g < kRowGroups; g++) {
            s0 += lred[2 * g];
            s1 += lred[2 * g + 1];
        }
        stat[2] = s0;
        stat[3] = s1;
    }

    // Thread t reduces output element (h = t / 128, d = t % 128) over the row groups.
    const int h = tid >> 7;
    const int d = tid & 127;
    float acc = 0.f;
#pragma unroll
    for (int g = 0; g < kRowGroups; g++) acc += red[((size_t)g * 2 + h) * kD + d];
    __syncthreads();  // stat[2..3] (the sums) are written
    const size_t out_head = (size_t)b * kHq * kD + (size_t)(kGroup * (kvh - a.kvh0)) * kD;

    if (nsplit == 1) {
        a.out[out_head + (size_t)h * kD + d] = acc / stat[2 + h];
        return;
    }

    float* recs = a.partials + (size_t)(b * kHkv + kvh) * a.nsplit_max * kRec;
    {
        float* mine = recs + (size_t)s * kRec;
        if (tid == 0) *reinterpret_cast<float4*>(mine) = make_float4(stat[0], stat[2], stat[1], stat[3]);
        mine[4 + h * kD + d] = acc;
    }
    // Publish the record, then take a ticket; the CTA that takes the last one merges.  One
    // thread takes the ticket with an acquire-release atomic on behalf of the CTA: the barrier
    // orders the other threads' record writes before its release, and its acquire makes the
    // other CTAs' records visible to the last CTA.
    __syncthreads();
    if (tid == 0) {
        unsigned int ticket;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                     : "=r"(ticket)
                     : "l"(&a.counters[b * kHkv + kvh])
                     : "memory");
        const int last = ticket == (unsigned int)(nsplit - 1);
        if (last) asm volatile("fence.proxy.async.global;" ::: "memory");  // records are read by TMA below
        *last_flag = last;
    }
    __syncthreads();
    if (!*last_flag) return;

    // ---- merge (last CTA of this sequence/KV head) -----------------------------------
    if (!merge_records(recs, nsplit, reinterpret_cast<float*>(kreg),
                       dec_k_region<T>(a.chunk) + dec_kv_bytes<T>(a.chunk), &bars[2], sc, a.out + out_head))
        return;
    if (tid == 0) a.counters[b * kHkv + kvh] = 0u;
}

// ---- BF16 single-sequence decode on the tensor cores ---------------------------------------
//
// Same split-KV scheme as decode_split_kernel, for one sequence with a BF16 cache, with the two
// contractions of a split on the tensor cores through warp-level mma.sync (m16n8k16, BF16 in,
// FP32 accumulate).  The contraction per split is tiny (2 query heads), so latency, not
// throughput, is what matters: one mma.sync replaces 256 scalar FMAs, a shuffle tree and the BF16
// unpacking of the CUDA-core form.  The FP32 query and the FP32 softmax weights enter as hi + lo
// BF16 pairs (x = hi + lo to 2^-16 relative), each pair two of the 8 columns of the B operand:
//   scores   S^T[rows][4] = K[rows][128] . [q0_hi q0_lo q1_hi q1_lo]^T,  s_h = S_h,hi + S_h,lo
//   output   O^T[128][4]  = V^T[128][rows] . [p0_hi p0_lo p1_hi p1_lo]^T, o_h = O_h,hi + O_h,lo
// (columns 4..7 are zero).  K and V tiles come by TMA tensor copies ({64 dims, chunk rows} boxes,
// 128-byte swizzle), so the A fragments load with ldmatrix free of bank conflicts.  The tensor
// maps span the whole slab (so they depend on the cache alone and are encoded once): tile rows
// past the attended rows hold whatever the slab has there -- masked out of the scores, and
// zeroed in the V tile.  Warps split the score rows by 16-row tiles and the output by 16-dim
// slices, so no cross-warp reduction of partial outputs is needed.  Split records and tickets
// are those of decode_split_kernel; the last CTA merges with plain loads from L2.

constexpr int kMmaMaxChunk = 256;    // rows per split (TMA boxes are at most 256 rows)
constexpr int kMmaBatchChunk = 192;  // rows per split for request batches
constexpr int kQaPitch = 272;  // bytes per A row of the query (256 + 16: conflict-free A loads)
// Warps per CTA (NW): the kernel is written for 8 or 16; 8 is the one launched (16 warps -- a score
// tile per warp, P.V in two row halves -- measured 4-7 % slower at 4K: more barrier and exchange
// cost than latency hidden).
constexpr int kMmaStat = 64 + 256;  // floats: block maxima and sums [16][2] x 2, P.V half exchange [8][2][16]

// ---- decode output gather over NVLink (KV-head sharding, one rank per GPU) -------------------
//
// With the KV heads of one sequence split over N ranks, every rank needs the whole [16][128]
// output of each decode call.  Instead of a separate collective per layer, the CTA that writes a
// head pair's final output also stores it into every rank's exchange buffer (peer stores over
// NVLink into memory mapped by CUDA IPC), each value as one 64-bit word that carries the call's
// epoch beside the value's bits: a word is single-copy atomic, so a reader that sees the epoch
// sees the value, and no fence or flag is needed.  The rank's last such CTA of the call (a
// device-scope ticket) then polls, bounded, the 16 x 128 words of its own buffer until each
// carries the epoch and writes the values to the caller -- inside the decode kernel, so a call is
// one launch.  Epochs (one per call, counted on each rank) grow by one per call, and the words
// are double-buffered by epoch parity: a rank can run at most one call ahead of another (its next
// call completes only once the other has stored its words of that call, which it does after
// completing the current one), so a word of two calls back is never taken for the current one.
// (The first form raised one flag per head after a system-scope release fence, ~2 us per call.)

constexpr int kGatherMaxRanks = 8;

struct GatherBuf {                          // one per rank, in that rank's device memory
    unsigned long long words[2][kHq][kD];   // by epoch parity: (epoch << 32) | the value's bits
    float stage[kHq][kD];                   // this rank's head pairs' outputs before they are sent
    unsigned int epoch;                     // calls this rank has completed (local)
    unsigned int done;                      // this rank's head pairs published in the current call
};

struct GatherDev {                          // device table, in this rank's memory
    GatherBuf* buf[kGatherMaxRanks];        // every rank's exchange buffer (peers through IPC)
    int rank;
    int world;
};

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p)
{
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_relaxed_sys(unsigned int* p, unsigned int v)
{
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v)
{
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Two words with one 16-byte load; each word is validated on its own (its epoch), so the pair
// need not be read at one instant.
__device__ __forceinline__ void ld_relaxed_sys_u64x2(const unsigned long long* p, unsigned long long& a,
                                                     unsigned long long& b)
{
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// Called by every thread of the CTA that has just written the rows of KV head kvh's query pair
// into this rank's stage: stores them, as epoch-carrying words, into slot epoch & 1 of every
// rank's buffer (its own included).  The rank's last head pair of the call (a device-scope
// ticket among this rank's CTAs) then reads all 16 x 128 words of its own slot, each polled until
// it carries the epoch (bounded: a rank that never publishes raises TYB_STATUS_WAIT_TIMEOUT), and
// writes the assembled [16][128] to `out`.
__device__ __forceinline__ void gather_publish(const GatherDev* g, int kvh, int nkvh_local, unsigned int epoch,
                                               float* out)
{
    __shared__ int s_last, s_fail;
    const int par = (int)(epoch & 1u);
    GatherBuf* mine = g->buf[g->rank];
    __syncthreads();  // the head pair's rows are in the stage
    if (threadIdx.x < 2 * kD) {
        const int i = kGroup * kvh * kD + threadIdx.x;  // element of [16][128]
        const unsigned long long w =
            ((unsigned long long)epoch << 32) | __float_as_uint((&mine->stage[0][0])[i]);
        for (int p = 0; p < g->world; p++) st_relaxed_sys_u64(&g->buf[p]->words[par][0][0] + i, w);
    }
    if (threadIdx.x == 0) {
        unsigned int t;
        asm volatile("atom.relaxed.gpu.global.add.u32 %0, [%1], 1;" : "=r"(t) : "l"(&mine->done) : "memory");
        s_last = t == (unsigned int)(nkvh_local - 1);
        if (s_last) mine->done = 0u;  // the next call's tickets come after this kernel has completed
        s_fail = 0;
    }
    __syncthreads();
    if (!s_last) return;
    // Each thread reads 8 consecutive words with all its loads in flight at once, then re-reads
    // until every one carries the epoch (polling one word at a time costs a round trip each).
    const unsigned long long* src = &mine->words[par][0][0];
    const uint64_t t0 = globaltimer_ns();
    for (int i0 = threadIdx.x * 8; i0 < kHq * kD; i0 += blockDim.x * 8) {
        unsigned long long w[8];
        bool all = false;
        while (!all) {
#pragma unroll
            for (int k = 0; k < 8; k += 2) ld_relaxed_sys_u64x2(src + i0 + k, w[k], w[k + 1]);
            all = true;
#pragma unroll
            for (int k = 0; k < 8; k++) all = all && (unsigned int)(w[k] >> 32) == epoch;
            if (!all && globaltimer_ns() - t0 > wait_limit_ns()) {
                raise_status(TYB_STATUS_WAIT_TIMEOUT);
                s_fail = 1;
                break;
            }
        }
        if (!all) break;
        float4* o = reinterpret_cast<float4*>(out + i0);
        o[0] = make_float4(__uint_as_float((unsigned int)w[0]), __uint_as_float((unsigned int)w[1]),
                           __uint_as_float((unsigned int)w[2]), __uint_as_float((unsigned int)w[3]));
        o[1] = make_float4(__uint_as_float((unsigned int)w[4]), __uint_as_float((unsigned int)w[5]),
                           __uint_as_float((unsigned int)w[6]), __uint_as_float((unsigned int)w[7]));
    }
    __syncthreads();
    if (threadIdx.x == 0 && !s_fail) mine->epoch = epoch;
}

struct DecodeMmaArgs {
    const float* q;  // [batch][16][128]
    float* out;      // query head 2 kvh0's row of sequence 0 (row stride 16 x 128 per sequence)
    // Request batch: per-sequence descriptors and tensor maps (K, V of sequence b at 2b, 2b + 1),
    // read after the dependency wait; NULL for one sequence (the fields below and the maps in
    // the parameters are used).
    const tyb_seq_kv* seqs;
    const CUtensorMap* maps;
    __nv_bfloat16* k;  // layer slab, head 0 (the new row is written through these)
    __nv_bfloat16* v;
    int row_capacity;
    int kv_len;
    const float* k_new;  // [8][128] fp32 row appended at kv_len - 1, or NULL
    const float* v_new;
    float scale_log2;
    int chunk;
    int nsplit;
    int prefetch_rows;
    float* partials;
    unsigned int* counters;
    int kvh0;
    int prefetch_small;
    int wide_counters;  // counters hold kHkv head counters then [kHkv][kGroupCounters] group counters
    const GatherDev* gather;  // non-NULL: outputs go to the exchange buffer and to every rank
    // Non-NULL q_norm: q and k_new arrive raw; RMSNorm(q_norm / k_norm, eps) and rotate_half
    // M-RoPE with the token's rope_cos / rope_sin [64] are applied on load (one sequence only).
    const float* q_norm;
    const float* k_norm;
    const float* rope_cos;
    const float* rope_sin;
    float eps;
};

__host__ __device__ constexpr size_t mma_pa_pitch(int chunk) { return (size_t)(chunk + 8) * 2; }

// [K tile chunk x 256 B][V tile][P rows 4 x pitch][q rows 4 x 272][stat kMmaStat floats]
// [3 mbarriers][flag], after rounding the base up to 1024 bytes (the swizzle repeats per 1 KB).
__host__ __device__ constexpr size_t decode_mma_smem_bytes(int chunk)
{
    return 1024 + (size_t)chunk * 512 + 4 * mma_pa_pitch(chunk) + 4 * kQaPitch + kMmaStat * sizeof(float) +
           3 * sizeof(uint64_t) + 16;
}

// QK-RMSNorm + rotate_half M-RoPE of one 128-dim row (kernel/ops.c:22-62 and :297-343, as
// kernel/decoder.c:73-93 applies them to q and k before the append and the attention):
// y = x * rsqrt(mean(x^2) + eps) * w, then z[j] = y[j] c[j] - y[j+64] s[j] and
// z[j+64] = y[j+64] c[j] + y[j] s[j] for j < 64.
// qk_prep_row4: the row as 4 consecutive values per lane over a full warp (lane l: dims 4l..4l+3).
__device__ __forceinline__ void qk_prep_row4(float (&x)[4], int lane, const float* w, const float* c,
                                             const float* sn, float eps)
{
    float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float rs = rsqrtf(ss * (1.f / kD) + eps);
    float y[4], partner[4];
#pragma unroll
    for (int e = 0; e < 4; e++) y[e] = x[e] * rs * w[4 * lane + e];
#pragma unroll
    for (int e = 0; e < 4; e++) partner[e] = __shfl_xor_sync(0xffffffffu, y[e], 16);
    const int j = (4 * lane) & 63;
#pragma unroll
    for (int e = 0; e < 4; e++)
        x[e] = lane < 16 ? y[e] * c[j + e] - partner[e] * sn[j + e] : y[e] * c[j + e] + partner[e] * sn[j + e];
}

// qk_prep_row8: the row as 8 consecutive values per lane over lanes 0-15 of a warp (lane i: dims
// 8i..8i+7); only those 16 lanes call it.
__device__ __forceinline__ void qk_prep_row8(float (&x)[8], int i, const float* w, const float* c,
                                             const float* sn, float eps)
{
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 8; e++) ss += x[e] * x[e];
#pragma unroll
    for (int o = 8; o >= 1; o >>= 1) ss += __shfl_xor_sync(0x0000ffffu, ss, o);
    const float rs = rsqrtf(ss * (1.f / kD) + eps);
    float y[8], partner[8];
#pragma unroll
    for (int e = 0; e < 8; e++) y[e] = x[e] * rs * w[8 * i + e];
#pragma unroll
    for (int e = 0; e < 8; e++) partner[e] = __shfl_xor_sync(0x0000ffffu, y[e], 8);
    const int j = (8 * i) & 63;
#pragma unroll
    for (int e = 0; e < 8; e++)
        x[e] = i < 8 ? y[e] * c[j + e] - partner[e] * sn[j + e] : y[e] * c[j + e] + partner[e] * sn[j + e];
}

__device__ __forceinline__ void mma_16816_full(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1)
{
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], uint32_t addr)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

// TMA tensor copy of the box at {c0 dims, c1 rows, c2 heads} into shared memory, on `bar`.
__device__ __forceinline__ void tma_box_3d(uint32_t smem_dst, const CUtensorMap* map, int c0, int c1, int c2,
                                           uint64_t* bar)
{
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
            "r"(smem_dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}

// Byte offset of dims [8 c16, 8 c16 + 8) of row r in a tile of `chunk` rows stored as two
// 64-dim halves with the 128-byte swizzle of the TMA copy (16-byte unit c ^ (r & 7)).
__device__ __forceinline__ uint32_t swz(int chunk, int r, int c16)
{
    return (uint32_t)((c16 >> 3) * chunk * 128 + r * 128 + (((c16 & 7) ^ (r & 7)) << 4));
}

__device__ __forceinline__ uint32_t pack_bf16_pair(float lo_elem, float hi_elem)
{
    __nv_bfloat162 h = __floats2bfloat162_rn(lo_elem, hi_elem);
    return *reinterpret_cast<uint32_t*>(&h);
}

// x ~ hi + lo in BF16 (hi = bf16(x), lo = bf16(x - hi)), for a pair of consecutive elements.
__device__ __forceinline__ void split_pair(float x0, float x1, uint32_t& hi, uint32_t& lo)
{
    const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
    const float2 hf = __bfloat1622float2(h);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = pack_bf16_pair(x0 - hf.x, x1 - hf.y);
}

// Merge of the `nsplit` split records of one KV head by the CTA that took the last ticket, with
// plain loads from L2 (no copy into shared memory; one load round trip per 32 records).  Per batch
// of 32: warp h (h = 0, 1) fetches the records' headers, one per lane, and computes head h's
// batch maximum, the rescale of what came before, each record's weight 2^(m_j - max) into `wts`
// and the running sum; meanwhile every thread fetches its element (h, d) = (tid / 128, tid % 128)
// of each record, then accumulates it against the weights with four independent chains.  Loads
// bypass L1 (.cg): the records were written by other CTAs, and the workspace by earlier launches.
// wts: 2 * 32 + 4 floats of shared memory.  Every thread of the CTA calls it; writes
// out[h * 128 + d].  step: records at recs + j * step * kRec.  rec_out non-NULL: the merge is
// written as a record instead (running maxima and sums in the header, O unnormalised), for a
// later merge of merges; it may be the first record read (all reads come first).
__device__ __forceinline__ void merge_records_direct(const float* recs, int nsplit, float* wts, float* out,
                                                     int step = 1, float* rec_out = nullptr)
{
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const bool active = tid < 2 * kD;  // threads past 256 only take part in the barriers
    const int h = (tid >> 7) & 1;
    const int d = tid & 127;
    float* alpha_s = wts + 64;  // [2] rescale of the running sums, [2] running weight sums
    float run = -INFINITY, Lrun = 0.f;  // warps 0, 1: head `warp`'s running maximum and sum
    float O = 0.f;
    for (int j0 = 0; j0 < nsplit; j0 += 32) {
        const int nb = min(32, nsplit - j0);
        const float* r = recs + (size_t)j0 * step * kRec;
        if (j0) __syncthreads();  // the previous batch's weights are consumed
        // Headers first: the weights (on the path to the output) need them.
        float mj = -INFINITY, lj = 0.f;
        if (warp < 2 && lane < nb) {
            const float2 e = __ldcg(reinterpret_cast<const float2*>(r + (size_t)lane * step * kRec + 2 * warp));
            mj = e.x;
            lj = e.y;
        }
        float ov[32];
#pragma unroll
        for (int j = 0; j < 32; j++) ov[j] = active && j < nb ? __ldcg(r + (size_t)j * step * kRec + 4 + h * kD + d) : 0.f;
        if (warp < 2) {
            float mb = mj;
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, off));
            const float nr = fmaxf(run, mb);
            const float alpha = fast_exp2(run - nr);  // 0 on the first batch
            const float w = lane < nb ? fast_exp2(mj - nr) : 0.f;
            float lw = w * lj;
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) lw += __shfl_xor_sync(0xffffffffu, lw, off);
            Lrun = Lrun * alpha + lw;
            run = nr;
            wts[32 * warp + lane] = w;
            if (lane == 0) {
                alpha_s[warp] = alpha;
                alpha_s[2 + warp] = Lrun;
            }
        }
        __syncthreads();
        if (active) {
            const float* wh = wts + 32 * h;
            float o4[4] = {O * alpha_s[h], 0.f, 0.f, 0.f};
#pragma unroll
            for (int j = 0; j < 32; j++) o4[j & 3] = fmaf(wh[j], ov[j], o4[j & 3]);  // w = 0 past nb
            O = (o4[0] + o4[1]) + (o4[2] + o4[3]);
        }
    }
    if (rec_out) {
        __syncthreads();  // every read of the records is done
        if (warp < 2 && lane == 0) {
            rec_out[2 * warp] = run;
            rec_out[2 * warp + 1] = Lrun;
        }
        if (active) rec_out[4 + (size_t)h * kD + d] = O;
        return;
    }
    if (active) out[(size_t)h * kD + d] = O / alpha_s[2 + h];
}

// Merge of a head's records when more than 64 CTAs share it (kGroupRecs-record groups, each
// merged into its first record by the group's last CTA -- the groups in parallel -- then the
// group records merged by the last group).  Returns true in the CTA that produced the output.
// Measured at 32K with one KV head (128 splits, one GPU, 28 layers): 234 us/step against 299 with
// one CTA merging all 128 records; with 64 records the one-CTA merge through shared memory wins.
// gcount: the head's group counters (zero between launches); hcount: its head counter.
constexpr int kGroupRecs = 16;
constexpr int kGroupCounters = 32;  // groups per head at most (512 records)
__device__ __forceinline__ bool merge_two_level(float* recs, int n, int s, float* wts, float* out,
                                                unsigned int* gcount, unsigned int* hcount, int* flag)
{
    const int tid = threadIdx.x;
    const int grp = s / kGroupRecs;
    const int gsize = min(kGroupRecs, n - grp * kGroupRecs);
    const int ngroups = (n + kGroupRecs - 1) / kGroupRecs;
    float* gfirst = recs + (size_t)grp * kGroupRecs * kRec;
    if (tid == 0) {
        unsigned int t;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(t) : "l"(&gcount[grp]) : "memory");
        *flag = t == (unsigned int)(gsize - 1);
    }
    __syncthreads();
    if (!*flag) return false;
    merge_records_direct(gfirst, gsize, wts, nullptr, 1, gfirst);
    __syncthreads();  // the group record is written
    if (tid == 0) {
        gcount[grp] = 0u;
        unsigned int t;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(t) : "l"(hcount) : "memory");
        *flag = t == (unsigned int)(ngroups - 1);
    }
    __syncthreads();
    if (!*flag) return false;
    merge_records_direct(recs, ngroups, wts, out, kGroupRecs);
    if (tid == 0) *hcount = 0u;
    return true;
}



// kQk: q and the new key row arrive raw and are normalised and rotated on load (DecodeMmaArgs).
template <int NW, bool kQk, typename In>
__global__ void __launch_bounds__(NW * 32, 16 / NW)
    decode_mma_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                      const __grid_constant__ CUtensorMap tmk16, const __grid_constant__ CUtensorMap tmv16,
                      const DecodeMmaArgs a, const __grid_constant__ In in)
{
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int s = blockIdx.x;
    const int kvh = a.kvh0 + blockIdx.y;
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int g = lane >> 2;  // fragment row group
    const int t = lane & 3;   // thread in group
    const int chunk = a.chunk;

    unsigned char* Kt = smem;
    unsigned char* Vt = smem + (size_t)chunk * 256;
    unsigned char* Pa = Vt + (size_t)chunk * 256;
    const int ppitch = (int)mma_pa_pitch(chunk);
    unsigned char* Qa = Pa + 4 * ppitch;
    float* stat = reinterpret_cast<float*>(Qa + 4 * kQaPitch);  // wmax[16][2] lw[16][2] xo[8][2][16]
    uint64_t* bars = reinterpret_cast<uint64_t*>(stat + kMmaStat);  // K, V, merge records
    int* last_flag = reinterpret_cast<int*>(bars + 3);
    const uint32_t kt_u32 = smem_u32(Kt), vt_u32 = smem_u32(Vt);

    const int b = blockIdx.z;
    const float* q_src = a.q;
    const float* k_src = a.k_new;
    const float* v_src = a.v_new;
    inline_inputs(in, q_src, k_src, v_src);
    const float* qb = q_src + (size_t)b * kHq * kD;
    int kv_len = a.kv_len;
    int nsplit = a.nsplit;
    const CUtensorMap* mk = &tmk;
    const CUtensorMap* mv = &tmv;
    const int r0 = s * chunk;
    int nrows = 0, trows = 0;
    auto geometry = [&]() {
        nrows = min(chunk, kv_len - r0);                       // >= 1 for a split that runs
        const int cache_rows = a.k_new ? kv_len - 1 : kv_len;  // rows read from the cache
        trows = max(0, min(nrows, cache_rows - r0));
    };
    bool early = false;
    if (!a.seqs) {
        geometry();
        early = r0 + trows <= a.prefetch_rows;
    }

    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        mbar_init(&bars[2], 1);
        fence_barrier_init();
        fence_proxy_async_smem();
    }
    __syncthreads();
    auto issue = [&]() {  // full boxes (rows past the slab arrive as zeros and count)
        const uint32_t half = (uint32_t)chunk * 128;
        if (!a.seqs && s == nsplit - 1 && nrows <= 64 && nrows < chunk) {
            // Short last split of one sequence: only the (at most 4) 16-row groups it attends,
            // with the 16-row maps (the same swizzle, since each group starts at a multiple of 16
            // rows); longer last splits take the full box (fewer copies to issue).
            const int groups = (nrows + 15) >> 4;
            mbar_arrive_expect_tx(&bars[0], (uint32_t)groups * 4096u);
            for (int i = 0; i < groups; i++) {
                tma_box_3d(kt_u32 + i * 2048, &tmk16, 0, r0 + 16 * i, kvh, &bars[0]);
                tma_box_3d(kt_u32 + half + i * 2048, &tmk16, 64, r0 + 16 * i, kvh, &bars[0]);
            }
            mbar_arrive_expect_tx(&bars[1], (uint32_t)groups * 4096u);
            for (int i = 0; i < groups; i++) {
                tma_box_3d(vt_u32 + i * 2048, &tmv16, 0, r0 + 16 * i, kvh, &bars[1]);
                tma_box_3d(vt_u32 + half + i * 2048, &tmv16, 64, r0 + 16 * i, kvh, &bars[1]);
            }
            return;
        }
        mbar_arrive_expect_tx(&bars[0], 2 * half);
        tma_box_3d(kt_u32, mk, 0, r0, kvh, &bars[0]);
        tma_box_3d(kt_u32 + half, mk, 64, r0, kvh, &bars[0]);
        mbar_arrive_expect_tx(&bars[1], 2 * half);
        tma_box_3d(vt_u32, mv, 0, r0, kvh, &bars[1]);
        tma_box_3d(vt_u32 + half, mv, 64, r0, kvh, &bars[1]);
    };
    if (tid == 0 && early) issue();
    const bool has_new = !a.seqs && a.k_new && kv_len - 1 >= r0 && kv_len - 1 < r0 + nrows;
    // q and the appended row may be written by the previous kernel: read after the wait, but
    // their L2 lines requested now (plain prefetches, one 128-byte line per lane).
    if (!kIsInline<In> && a.prefetch_small && warp == 1) {
        const float* line = nullptr;
        if (lane < 8)
            line = qb + (size_t)(kGroup * kvh) * kD + lane * 32;
        else if (lane < 16 && has_new)
            line = (lane < 12 ? k_src : v_src) + (size_t)kvh * kD + (lane & 3) * 32;
        if (line) asm volatile("prefetch.global.L2 [%0];" ::"l"(line));
    }
    pdl_wait();
    pdl_trigger();
    if (a.seqs) {
        // Request batch: this sequence's geometry and tensor maps (written before the launch).
        const tyb_seq_kv d = a.seqs[b];
        kv_len = d.kv_len;
        nsplit = (kv_len + chunk - 1) / chunk;
        if (s >= nsplit) return;
        geometry();
        mk = a.maps + 2 * b;
        mv = mk + 1;
        if (tid == 0) {
            asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(mk) : "memory");
            asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(mv) : "memory");
        }
    }
    if (tid == 0 && !early) issue();

    // The query of both heads as A rows q0_hi, q0_lo, q1_hi, q1_lo (BF16).
    if (tid < 64) {
        const int h = tid >> 5, d0 = (tid & 31) * 4;
        float4 x = *reinterpret_cast<const float4*>(qb + (size_t)(kGroup * kvh + h) * kD + d0);
        if (kQk) {  // raw query: RMSNorm + M-RoPE here (warp = one head, lane = 4 dims)
            float v4[4] = {x.x, x.y, x.z, x.w};
            qk_prep_row4(v4, tid & 31, a.q_norm, a.rope_cos, a.rope_sin, a.eps);
            x = make_float4(v4[0], v4[1], v4[2], v4[3]);
        }
        uint32_t hi0, lo0, hi1, lo1;
        split_pair(x.x, x.y, hi0, lo0);
        split_pair(x.z, x.w, hi1, lo1);
        *reinterpret_cast<uint2*>(Qa + (2 * h) * kQaPitch + d0 * 2) = make_uint2(hi0, hi1);
        *reinterpret_cast<uint2*>(Qa + (2 * h + 1) * kQaPitch + d0 * 2) = make_uint2(lo0, lo1);
    }
    // The appended row: threads 64..79 write it to the cache and, once the tiles have landed,
    // into its tile row (the copy may have read the slab's old contents there).
    const int rn = kv_len - 1 - r0;
    const bool new_thread = has_new && tid >= 64 && tid < 80;
    float nk[8], nv[8];
    if (new_thread) {
        const int i = tid - 64;
        const size_t off = (size_t)kvh * kD + i * 8;
        load8(k_src + off, nk);
        load8(v_src + off, nv);
        if (kQk) qk_prep_row8(nk, i, a.k_norm, a.rope_cos, a.rope_sin, a.eps);  // raw k: normed, rotated
        const size_t row = ((size_t)kvh * a.row_capacity + (kv_len - 1)) * kD + i * 8;
        store8(a.k + row, nk);
        store8(a.v + row, nv);
    }
    const bool kok = mbar_wait_bounded(&bars[0], 0, wait_limit_ns(), TYB_STATUS_WAIT_TIMEOUT);
    if (new_thread) store8(reinterpret_cast<__nv_bfloat16*>(Kt + swz(chunk, rn, tid - 64)), nk);
    if (__syncthreads_or(!kok)) return;

    // Scores: S^T[16 rows][8] = K[16 rows][128] . [q0_hi q0_lo q1_hi q1_lo 0 0 0 0]^T per 16-row
    // tile (K rows as the A operand, ldmatrix from the swizzled tile; the query as the 8 B
    // columns, 4 of them zero).  Warp w takes tiles w and w + 8 of the first ceil16(nrows) rows.
    // In the accumulator, lane (g, t) holds rows g and g + 8 of columns 2t, 2t + 1: lanes with
    // t = h < 2 get s_h = column hi + column lo of both rows, with no data exchange.
    const int ntiles = (nrows + 15) >> 4;  // 16-row tiles
    uint32_t qb0[8], qb1[8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
        qb0[j] = 0u;
        qb1[j] = 0u;
        if (lane < 16) {
            qb0[j] = *reinterpret_cast<const uint32_t*>(Qa + g * kQaPitch + (16 * j + 2 * t) * 2);
            qb1[j] = *reinterpret_cast<const uint32_t*>(Qa + g * kQaPitch + (16 * j + 8 + 2 * t) * 2);
        }
    }
    constexpr int KT = 16 / NW;      // score tiles per warp
    constexpr int HALVES = NW / 8;   // row parts of P.V
    constexpr int STEPS = 16 / HALVES;  // 16-row steps per part
    const bool holder = t < 2;  // head t
    const int arow = (lane & 7) + 8 * ((lane >> 3) & 1);
    const int acol = lane >> 4;
    // Warp w scores tiles w, w + NW, ...  All A fragments of a warp's tiles are loaded before the
    // first mma (ldmatrix takes ~50 cycles; loading each just before its mma would serialise them).
    float c[KT][2][4];  // [tile][even / odd 16-dim step]
#pragma unroll
    for (int k = 0; k < KT; k++)
#pragma unroll
        for (int e = 0; e < 4; e++) c[k][0][e] = c[k][1][e] = 0.f;
    {
        uint32_t af[KT][8][4];
#pragma unroll
        for (int k = 0; k < KT; k++)
            if (warp + NW * k < ntiles)
#pragma unroll
                for (int j = 0; j < 8; j++)
                    ldsm_x4(af[k][j], kt_u32 + swz(chunk, (warp + NW * k) * 16 + arow, 2 * j + acol));
#pragma unroll
        for (int k = 0; k < KT; k++)
            if (warp + NW * k < ntiles)
#pragma unroll
                for (int j = 0; j < 8; j++) mma_16816_full(c[k][j & 1], af[k][j], qb0[j], qb1[j]);
    }
    float sv[KT][2];  // [tile][row g, row g + 8]
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < KT; k++) {
        const int rb = (warp + NW * k) * 16 + g;
        const bool live = warp + NW * k < ntiles;
        const float s0 = c[k][0][0] + c[k][1][0] + c[k][0][1] + c[k][1][1];
        const float s1 = c[k][0][2] + c[k][1][2] + c[k][0][3] + c[k][1][3];
        sv[k][0] = live && rb < nrows ? s0 * a.scale_log2 : -INFINITY;
        sv[k][1] = live && rb + 8 < nrows ? s1 * a.scale_log2 : -INFINITY;
        m = fmaxf(m, fmaxf(sv[k][0], sv[k][1]));
    }
    // Maximum over the warp's rows: lanes of equal t.
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
    float* wmax = stat;     // [NW warps][2]
    float* lw = stat + 32;  // [NW warps][2]
    float* xo = stat + 64;  // [8 dim slices][2 heads][16 dims]
    if (lane < 2) wmax[2 * warp + lane] = m;
    __syncthreads();
    const int hh = t & 1;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; w++) M = fmaxf(M, wmax[2 * w + hh]);

    // Weights: p = 2^(s - M), written as P rows p0_hi, p0_lo, p1_hi, p1_lo; sums per warp.
    float l = 0.f;
#pragma unroll
    for (int k = 0; k < KT; k++) {
        if (holder && warp + NW * k < ntiles) {
            const int rb = (warp + NW * k) * 16 + g;
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const float p = fast_exp2(sv[k][u] - M);
                l += p;
                const __nv_bfloat16 hi = __float2bfloat16_rn(p);
                const __nv_bfloat16 lo = __float2bfloat16_rn(p - __bfloat162float(hi));
                *reinterpret_cast<__nv_bfloat16*>(Pa + (2 * hh) * ppitch + (rb + 8 * u) * 2) = hi;
                *reinterpret_cast<__nv_bfloat16*>(Pa + (2 * hh + 1) * ppitch + (rb + 8 * u) * 2) = lo;
            }
        }
    }
    l += __shfl_xor_sync(0xffffffffu, l, 4);
    l += __shfl_xor_sync(0xffffffffu, l, 8);
    l += __shfl_xor_sync(0xffffffffu, l, 16);
    if (lane < 2) lw[2 * warp + lane] = l;

    const bool vok = mbar_wait_bounded(&bars[1], 0, wait_limit_ns(), TYB_STATUS_WAIT_TIMEOUT);
    // V rows the weights do not cover but the last 16-row step reads: zeros (0 * stale NaN is NaN).
    {
        const int z0 = trows + (has_new ? 1 : 0), z1 = ntiles * 16;
        for (int i = tid; i < (z1 - z0) * 16; i += NW * 32)
            *reinterpret_cast<uint4*>(Vt + swz(chunk, z0 + (i >> 4), i & 15)) = make_uint4(0u, 0u, 0u, 0u);
    }
    if (new_thread) store8(reinterpret_cast<__nv_bfloat16*>(Vt + swz(chunk, rn, tid - 64)), nv);
    if (__syncthreads_or(!vok)) return;

    // Output: O^T[16 dims][8] = V^T[16 dims][rows] . [p0_hi p0_lo p1_hi p1_lo 0 0 0 0]^T.  Warp w
    // owns dims [16 (w % 8), + 16) of row part w / 8 (steps STEPS part .. + STEPS - 1; V^T
    // fragments by transposing ldmatrix), two accumulators (even and odd steps); with two parts
    // the second part's partial outputs go through shared memory to the first.  Lane (g, t < 2)
    // ends with head t's dims 16 (w % 8) + g, + 8.
    const int slice = warp & 7;
    const int half = warp >> 3;
    float o[2][4];
#pragma unroll
    for (int e = 0; e < 4; e++) o[0][e] = o[1][e] = 0.f;
    {
        const int vrow = (lane & 7) + 8 * (lane >> 4);
        const int vcol = 2 * slice + ((lane >> 3) & 1);
        // Groups of 4 steps (fragments of a group loaded, then its mma), the loop unrolled so
        // that a group's loads are issued while the previous group's mma run: 186.7 against
        // 191.6 us per decode step at 4K with the loop kept rolled (measured; all 16 steps'
        // fragments loaded up front, or groups of 2 or 8, were slower than rolled groups of 4).
#pragma unroll
        for (int i0 = 0; i0 < STEPS; i0 += 4) {
            uint32_t va[4][4], pb[4][2];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int j = STEPS * half + i0 + i;
                if (j < ntiles) {
                    pb[i][0] = pb[i][1] = 0u;
                    if (lane < 16) {
                        const unsigned char* row = Pa + g * ppitch + (16 * j + 2 * t) * 2;
                        pb[i][0] = *reinterpret_cast<const uint32_t*>(row);
                        pb[i][1] = *reinterpret_cast<const uint32_t*>(row + 16);
                    }
                    ldsm_x4_trans(va[i], vt_u32 + swz(chunk, 16 * j + vrow, vcol));
                }
            }
#pragma unroll
            for (int i = 0; i < 4; i++)
                if (STEPS * half + i0 + i < ntiles) mma_16816_full(o[i & 1], va[i], pb[i][0], pb[i][1]);
        }
    }
    float y0 = o[0][0] + o[1][0] + o[0][1] + o[1][1];  // dim 16 slice + g
    float y1 = o[0][2] + o[1][2] + o[0][3] + o[1][3];  // dim 16 slice + g + 8
    const bool writer = half == 0 && holder;  // the first part's warps write the result
    if (HALVES > 1) {
        if (half && holder) {
            xo[(slice * 2 + hh) * 16 + g] = y0;
            xo[(slice * 2 + hh) * 16 + g + 8] = y1;
        }
        __syncthreads();
        if (writer) {
            y0 += xo[(slice * 2 + hh) * 16 + g];
            y1 += xo[(slice * 2 + hh) * 16 + g + 8];
        }
    }
    float L = 0.f;
#pragma unroll
    for (int w = 0; w < NW; w++) L += lw[2 * w + hh];
    const int dim = 16 * slice + g;
    // rows of query heads 2 kvh, 2 kvh + 1 of sequence b (or of this rank's exchange slot)
    unsigned int epoch = 0;
    float* out_pair = a.out + (size_t)b * kHq * kD + (size_t)(kGroup * (kvh - a.kvh0)) * kD;
    if (a.gather) {
        epoch = __ldcg(&a.gather->buf[a.gather->rank]->epoch) + 1u;
        out_pair = &a.gather->buf[a.gather->rank]->stage[kGroup * kvh][0];
    }

    if (nsplit == 1) {
        if (writer) {
            float* o_ = out_pair + (size_t)hh * kD + dim;
            const float inv = 1.f / L;
            o_[0] = y0 * inv;
            o_[8] = y1 * inv;
        }
        if (a.gather) gather_publish(a.gather, kvh, gridDim.y, epoch, a.out);
        return;
    }

    float* recs = a.partials + ((size_t)b * kHkv + kvh) * a.nsplit * kRec;  // a.nsplit: the record stride
    {
        float* mine = recs + (size_t)s * kRec;
        if (writer) {
            float* o_ = mine + 4 + (size_t)hh * kD + dim;
            o_[0] = y0;
            o_[8] = y1;
            if (g == 0 && warp == 0) {
                mine[2 * hh] = M;
                mine[2 * hh + 1] = L;
            }
        }
    }
    __syncthreads();
    if (a.wide_counters && !a.seqs && nsplit > 64) {  // many splits of one sequence's head: merged in two levels
        if (!merge_two_level(recs, nsplit, s, reinterpret_cast<float*>(Kt), out_pair,
                             a.counters + kHkv + (size_t)kvh * kGroupCounters, &a.counters[kvh], last_flag))
            return;
        if (a.gather) gather_publish(a.gather, kvh, gridDim.y, epoch, a.out);
        return;
    }
    if (tid == 0) {
        unsigned int ticket;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                     : "=r"(ticket)
                     : "l"(&a.counters[b * kHkv + kvh])
                     : "memory");
        *last_flag = ticket == (unsigned int)(nsplit - 1);
        if (*last_flag && nsplit > 32) asm volatile("fence.proxy.async.global;" ::: "memory");  // read by a bulk copy
    }
    __syncthreads();
    if (!*last_flag) return;
    // Up to 32 records: plain L2 loads, one round trip.  More (sequences split over 33-128 CTAs per
    // KV head, as when one long sequence's heads are spread over GPUs): one bulk copy of the
    // records into the CTA's free tile space and the merge from shared memory -- a round trip
    // per 32 records measured ~1.4 us each.
    if (nsplit > 32) {
        if (!merge_records(recs, nsplit, reinterpret_cast<float*>(Kt), (size_t)(Qa - Kt), &bars[2], stat, out_pair))
            return;
    } else {
        merge_records_direct(recs, nsplit, reinterpret_cast<float*>(Kt), out_pair);
    }
    if (tid == 0) a.counters[b * kHkv + kvh] = 0u;
    if (a.gather) gather_publish(a.gather, kvh, gridDim.y, epoch, a.out);
}

// ---- streaming form: many waves (request batches, long sequences) ----------------------------
//
// When the splits of a launch cannot all be resident at once, each CTA instead walks a span of
// rows of one (sequence, KV head) in 96-row stages: the K and V tiles of stage s + 2 are requested
// (TMA tensor copies, 128-byte swizzle) while stage s is computed from the other buffer, with an
// online softmax across stages (running maximum per head, the output accumulators rescaled in
// registers).  The contractions are those of decode_mma_kernel (mma.sync, hi/lo BF16 query and
// weights); one record per span, merged by the span that takes the last ticket.  Two CTAs per SM
// (100 KB of shared memory each).  Measured alternatives: 64-row stages at three CTAs per SM and
// 128-row stages at one: 18-22 % slower on the 64-sequence batch (config 4).

constexpr int kStRows = 96;                         // rows per stage
constexpr size_t kStTile = (size_t)kStRows * 256;   // bytes of a K (or V) stage tile
constexpr int kStPitch = (kStRows + 8) * 2;         // bytes per P row (conflict-free B loads)

__host__ __device__ constexpr size_t decode_stream_smem_bytes()
{
    return 1024 + 4 * kStTile + 4 * kStPitch + 4 * kQaPitch + 32 * sizeof(float) + 5 * sizeof(uint64_t) + 16;
}

template <bool kQk, typename In>  // as in decode_mma_kernel
__global__ void __launch_bounds__(256, 2)
    decode_stream_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                         const DecodeMmaArgs a, const __grid_constant__ In in)
{
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int span = blockIdx.x;
    const int kvh = a.kvh0 + blockIdx.y;
    const int b = blockIdx.z;
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int g = lane >> 2;
    const int t = lane & 3;

    unsigned char* Pa = smem + 4 * kStTile;
    unsigned char* Qa = Pa + 4 * kStPitch;
    float* stat = reinterpret_cast<float*>(Qa + 4 * kQaPitch);  // wmax[8][2] lw[8][2]
    uint64_t* bars = reinterpret_cast<uint64_t*>(stat + 32);    // K0 K1 V0 V1 merge
    int* last_flag = reinterpret_cast<int*>(bars + 5);
    const uint32_t base_u32 = smem_u32(smem);  // K0 K1 V0 V1 tiles, kStTile apart

    const float* q_src = a.q;
    const float* k_src = a.k_new;
    const float* v_src = a.v_new;
    inline_inputs(in, q_src, k_src, v_src);
    const float* qb = q_src + (size_t)b * kHq * kD;
    int kv_len = a.kv_len;
    const CUtensorMap* mk = &tmk;
    const CUtensorMap* mv = &tmv;

    if (tid == 0) {
#pragma unroll
        for (int i = 0; i < 5; i++) mbar_init(&bars[i], 1);
        fence_barrier_init();
        fence_proxy_async_smem();
    }
    __syncthreads();
    if (!kIsInline<In> && a.prefetch_small && warp == 1 && lane < 8)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(qb + (size_t)(kGroup * kvh) * kD + lane * 32));
    // One sequence: the tiles of the first two stages are requested before the dependency wait
    // when the previous kernel wrote none of their cache rows (rows of a box past them are masked
    // out, zeroed, or -- the appended row -- replaced in shared memory).
    int early_st = 0;
    if (!a.seqs && tid == 0) {
        const int rb = span * a.chunk;
        if (rb < a.kv_len) {
            const int re = min(a.kv_len, rb + a.chunk);
            const int ns = (re - rb + kStRows - 1) / kStRows;
            const int crows = a.k_new ? a.kv_len - 1 : a.kv_len;
            for (int st = 0; st < min(2, ns); st++) {
                if (min(crows, min(re, rb + (st + 1) * kStRows)) > a.prefetch_rows) break;
                const uint32_t dk = base_u32 + (uint32_t)(st * kStTile), dv = base_u32 + (uint32_t)((2 + st) * kStTile);
                mbar_arrive_expect_tx(&bars[st], (uint32_t)kStTile);
                tma_box_3d(dk, &tmk, 0, rb + st * kStRows, kvh, &bars[st]);
                tma_box_3d(dk + (uint32_t)(kStTile / 2), &tmk, 64, rb + st * kStRows, kvh, &bars[st]);
                mbar_arrive_expect_tx(&bars[2 + st], (uint32_t)kStTile);
                tma_box_3d(dv, &tmv, 0, rb + st * kStRows, kvh, &bars[2 + st]);
                tma_box_3d(dv + (uint32_t)(kStTile / 2), &tmv, 64, rb + st * kStRows, kvh, &bars[2 + st]);
                early_st = st + 1;
            }
        }
    }
    pdl_wait();
    pdl_trigger();
    if (a.seqs) {
        const tyb_seq_kv d = a.seqs[b];
        kv_len = d.kv_len;
        mk = a.maps + 2 * b;
        mv = mk + 1;
        if (tid == 0) {
            asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(mk) : "memory");
            asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(mv) : "memory");
        }
    }
    const int r_begin = span * a.chunk;  // a.chunk: rows per span (a multiple of kStRows)
    if (r_begin >= kv_len) return;
    const int r_end = min(kv_len, r_begin + a.chunk);
    const int nst = (r_end - r_begin + kStRows - 1) / kStRows;
    const int nspan = (kv_len + a.chunk - 1) / a.chunk;
    const bool append = !a.seqs && a.k_new;
    const int cache_rows = append ? kv_len - 1 : kv_len;

    auto issue_k = [&](int st) {
        const int buf = st & 1;
        const uint32_t dst = base_u32 + (uint32_t)(buf * kStTile);
        mbar_arrive_expect_tx(&bars[buf], (uint32_t)kStTile);
        tma_box_3d(dst, mk, 0, r_begin + st * kStRows, kvh, &bars[buf]);
        tma_box_3d(dst + (uint32_t)(kStTile / 2), mk, 64, r_begin + st * kStRows, kvh, &bars[buf]);
    };
    auto issue_v = [&](int st) {
        const int buf = st & 1;
        const uint32_t dst = base_u32 + (uint32_t)((2 + buf) * kStTile);
        mbar_arrive_expect_tx(&bars[2 + buf], (uint32_t)kStTile);
        tma_box_3d(dst, mv, 0, r_begin + st * kStRows, kvh, &bars[2 + buf]);
        tma_box_3d(dst + (uint32_t)(kStTile / 2), mv, 64, r_begin + st * kStRows, kvh, &bars[2 + buf]);
    };
    if (tid == 0) {
        for (int st = early_st; st < min(2, nst); st++) {
            issue_k(st);
            issue_v(st);
        }
    }

    // The query as B columns q0_hi, q0_lo, q1_hi, q1_lo; the appended row to the cache.
    if (tid < 64) {
        const int h = tid >> 5, d0 = (tid & 31) * 4;
        float4 x = *reinterpret_cast<const float4*>(qb + (size_t)(kGroup * kvh + h) * kD + d0);
        if (kQk) {  // raw query: RMSNorm + M-RoPE here (warp = one head, lane = 4 dims)
            float v4[4] = {x.x, x.y, x.z, x.w};
            qk_prep_row4(v4, tid & 31, a.q_norm, a.rope_cos, a.rope_sin, a.eps);
            x = make_float4(v4[0], v4[1], v4[2], v4[3]);
        }
        uint32_t hi0, lo0, hi1, lo1;
        split_pair(x.x, x.y, hi0, lo0);
        split_pair(x.z, x.w, hi1, lo1);
        *reinterpret_cast<uint2*>(Qa + (2 * h) * kQaPitch + d0 * 2) = make_uint2(hi0, hi1);
        *reinterpret_cast<uint2*>(Qa + (2 * h + 1) * kQaPitch + d0 * 2) = make_uint2(lo0, lo1);
    }
    const bool new_here_span = append && kv_len - 1 >= r_begin && kv_len - 1 < r_end;
    const bool new_thread = new_here_span && tid >= 64 && tid < 80;
    float nk[8], nv[8];
    if (new_thread) {
        const int i = tid - 64;
        const size_t off = (size_t)kvh * kD + i * 8;
        load8(k_src + off, nk);
        load8(v_src + off, nv);
        if (kQk) qk_prep_row8(nk, i, a.k_norm, a.rope_cos, a.rope_sin, a.eps);  // raw k: normed, rotated
        const size_t row = ((size_t)kvh * a.row_capacity + (kv_len - 1)) * kD + i * 8;
        store8(a.k + row, nk);
        store8(a.v + row, nv);
    }
    __syncthreads();
    uint32_t qb0[8], qb1[8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
        qb0[j] = 0u;
        qb1[j] = 0u;
        if (lane < 16) {
            qb0[j] = *reinterpret_cast<const uint32_t*>(Qa + g * kQaPitch + (16 * j + 2 * t) * 2);
            qb1[j] = *reinterpret_cast<const uint32_t*>(Qa + g * kQaPitch + (16 * j + 8 + 2 * t) * 2);
        }
    }

    const bool holder = t < 2;
    const int hh = t & 1;  // head of this lane's accumulator columns (holders)
    const int arow = (lane & 7) + 8 * ((lane >> 3) & 1);
    const int acol = lane >> 4;
    const int vrow = (lane & 7) + 8 * (lane >> 4);
    const int vcol = 2 * warp + ((lane >> 3) & 1);
    float* wmax = stat;
    float* lw = stat + 16;
    float Mrun = -INFINITY, Lrun = 0.f;  // head hh
    float o[2][4];
#pragma unroll
    for (int e = 0; e < 4; e++) o[0][e] = o[1][e] = 0.f;

    for (int st = 0; st < nst; st++) {
        const int buf = st & 1;
        const uint32_t par = (uint32_t)((st >> 1) & 1);
        const uint32_t kt_u32 = base_u32 + (uint32_t)(buf * kStTile);
        const uint32_t vt_u32 = base_u32 + (uint32_t)((2 + buf) * kStTile);
        const int r0 = r_begin + st * kStRows;
        const int nrows = min(kStRows, r_end - r0);
        const int ntiles = (nrows + 15) >> 4;
        const int trows = max(0, min(nrows, cache_rows - r0));
        const bool new_here = append && kv_len - 1 >= r0 && kv_len - 1 < r0 + nrows;
        const int rn = kv_len - 1 - r0;

        const bool kok = mbar_wait_bounded(&bars[buf], par, wait_limit_ns(), TYB_STATUS_WAIT_TIMEOUT);
        if (new_here && new_thread)
            store8(reinterpret_cast<__nv_bfloat16*>(smem + buf * kStTile + swz(kStRows, rn, tid - 64)), nk);
        if (__syncthreads_or(!kok)) return;

        // Scores of tile w (warp w < ntiles), rows g and g + 8.
        float c[2][4];
#pragma unroll
        for (int e = 0; e < 4; e++) c[0][e] = c[1][e] = 0.f;
        if (warp < ntiles) {
            uint32_t af[8][4];
#pragma unroll
            for (int j = 0; j < 8; j++) ldsm_x4(af[j], kt_u32 + swz(kStRows, warp * 16 + arow, 2 * j + acol));
#pragma unroll
            for (int j = 0; j < 8; j++) mma_16816_full(c[j & 1], af[j], qb0[j], qb1[j]);
        }
        const int rb = warp * 16 + g;
        const float sv0 = warp < ntiles && rb < nrows ? (c[0][0] + c[1][0] + c[0][1] + c[1][1]) * a.scale_log2
                                                      : -INFINITY;
        const float sv1 = warp < ntiles && rb + 8 < nrows ? (c[0][2] + c[1][2] + c[0][3] + c[1][3]) * a.scale_log2
                                                          : -INFINITY;
        float m = fmaxf(sv0, sv1);
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
        if (lane < 2) wmax[2 * warp + lane] = m;
        __syncthreads();
        if (tid == 0 && st + 2 < nst) issue_k(st + 2);  // this K buffer is read no more
        float mst = -INFINITY;
#pragma unroll
        for (int w = 0; w < 8; w++) mst = fmaxf(mst, wmax[2 * w + hh]);
        const float Mnew = fmaxf(Mrun, mst);
        const float alpha = fast_exp2(Mrun - Mnew);  // 0 on the first stage

        float l = 0.f;
        if (holder && warp < ntiles) {
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const float p = fast_exp2((u ? sv1 : sv0) - Mnew);
                l += p;
                const __nv_bfloat16 hi = __float2bfloat16_rn(p);
                const __nv_bfloat16 lo = __float2bfloat16_rn(p - __bfloat162float(hi));
                *reinterpret_cast<__nv_bfloat16*>(Pa + (2 * hh) * kStPitch + (rb + 8 * u) * 2) = hi;
                *reinterpret_cast<__nv_bfloat16*>(Pa + (2 * hh + 1) * kStPitch + (rb + 8 * u) * 2) = lo;
            }
        }
        l += __shfl_xor_sync(0xffffffffu, l, 4);
        l += __shfl_xor_sync(0xffffffffu, l, 8);
        l += __shfl_xor_sync(0xffffffffu, l, 16);
        if (lane < 2) lw[2 * warp + lane] = l;

        const bool vok = mbar_wait_bounded(&bars[2 + buf], par, wait_limit_ns(), TYB_STATUS_WAIT_TIMEOUT);
        {
            // Tile rows past the attended ones that the last 16-row step reads: zeros.
            const int z0 = trows + (new_here ? 1 : 0), z1 = ntiles * 16;
            for (int i = tid; i < (z1 - z0) * 16; i += 256)
                *reinterpret_cast<uint4*>(smem + (2 + buf) * kStTile + swz(kStRows, z0 + (i >> 4), i & 15)) =
                    make_uint4(0u, 0u, 0u, 0u);
        }
        if (new_here && new_thread)
            store8(reinterpret_cast<__nv_bfloat16*>(smem + (2 + buf) * kStTile + swz(kStRows, rn, tid - 64)), nv);
        if (__syncthreads_or(!vok)) return;

        // O^T for the warp's 16 dims, rescaled to the new maximum first.
#pragma unroll
        for (int e = 0; e < 4; e++) {
            o[0][e] *= alpha;
            o[1][e] *= alpha;
        }
        {
            uint32_t va[kStRows / 16][4], pb[kStRows / 16][2];
#pragma unroll
            for (int i = 0; i < kStRows / 16; i++) {
                if (i < ntiles) {
                    pb[i][0] = pb[i][1] = 0u;
                    if (lane < 16) {
                        const unsigned char* row = Pa + g * kStPitch + (16 * i + 2 * t) * 2;
                        pb[i][0] = *reinterpret_cast<const uint32_t*>(row);
                        pb[i][1] = *reinterpret_cast<const uint32_t*>(row + 16);
                    }
                    ldsm_x4_trans(va[i], vt_u32 + swz(kStRows, 16 * i + vrow, vcol));
                }
            }
#pragma unroll
            for (int i = 0; i < kStRows / 16; i++)
                if (i < ntiles) mma_16816_full(o[i & 1], va[i], pb[i][0], pb[i][1]);
        }
        float lsum = 0.f;
#pragma unroll
        for (int w = 0; w < 8; w++) lsum += lw[2 * w + hh];
        Lrun = Lrun * alpha + lsum;
        Mrun = Mnew;
        __syncthreads();  // this V buffer, P, and the per-warp maxima and sums are read no more
        if (tid == 0 && st + 2 < nst) issue_v(st + 2);
    }

    const float y0 = o[0][0] + o[1][0] + o[0][1] + o[1][1];  // dim 16 warp + g, head hh (holders)
    const float y1 = o[0][2] + o[1][2] + o[0][3] + o[1][3];  // dim 16 warp + g + 8
    const int dim = 16 * warp + g;
    unsigned int epoch = 0;
    float* out_pair = a.out + (size_t)b * kHq * kD + (size_t)(kGroup * (kvh - a.kvh0)) * kD;
    if (a.gather) {
        epoch = __ldcg(&a.gather->buf[a.gather->rank]->epoch) + 1u;
        out_pair = &a.gather->buf[a.gather->rank]->stage[kGroup * kvh][0];
    }
    if (nspan == 1) {
        if (holder) {
            float* o_ = out_pair + (size_t)hh * kD + dim;
            const float inv = 1.f / Lrun;
            o_[0] = y0 * inv;
            o_[8] = y1 * inv;
        }
        if (a.gather) gather_publish(a.gather, kvh, gridDim.y, epoch, a.out);
        return;
    }
    float* recs = a.partials + ((size_t)b * kHkv + kvh) * a.nsplit * kRec;  // a.nsplit: the record stride
    {
        float* mine = recs + (size_t)span * kRec;
        if (holder) {
            float* o_ = mine + 4 + (size_t)hh * kD + dim;
            o_[0] = y0;
            o_[8] = y1;
            if (g == 0 && warp == 0) {
                mine[2 * hh] = Mrun;
                mine[2 * hh + 1] = Lrun;
            }
        }
    }
    __syncthreads();
    if (a.wide_counters && !a.seqs && nspan > 64) {  // as in decode_mma_kernel
        if (!merge_two_level(recs, nspan, span, reinterpret_cast<float*>(smem), out_pair,
                             a.counters + kHkv + (size_t)kvh * kGroupCounters, &a.counters[kvh], last_flag))
            return;
        if (a.gather) gather_publish(a.gather, kvh, gridDim.y, epoch, a.out);
        return;
    }
    if (tid == 0) {
        unsigned int ticket;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                     : "=r"(ticket)
                     : "l"(&a.counters[b * kHkv + kvh])
                     : "memory");
        *last_flag = ticket == (unsigned int)(nspan - 1);
        if (*last_flag && nspan > 32) asm volatile("fence.proxy.async.global;" ::: "memory");  // read by a bulk copy
    }
    __syncthreads();
    if (!*last_flag) return;
    if (nspan > 32) {  // as in decode_mma_kernel: many records through shared memory
        if (!merge_records(recs, nspan, reinterpret_cast<float*>(smem), (size_t)(Qa - smem), &bars[4], stat, out_pair))
            return;
    } else {
        merge_records_direct(recs, nspan, reinterpret_cast<float*>(smem), out_pair);
    }
    if (tid == 0) a.counters[b * kHkv + kvh] = 0u;
    if (a.gather) gather_publish(a.gather, kvh, gridDim.y, epoch, a.out);
}

// ---- host-side planning ----------------------------------------------------------------

// Everything cached below (SM counts, occupancies, kernel attributes) is per device: one process
// may drive several GPUs, and function attributes belong to each device's context.
constexpr int kMaxDevices = 64;

static int cur_dev()
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) dev = 0;
    return dev;
}

static int g_num_sms[kMaxDevices];

static int num_sms()
{
    const int dev = cur_dev();
    if (!g_num_sms[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        g_num_sms[dev] = n;
    }
    return g_num_sms[dev];
}

template <typename T>
static int blocks_per_sm(int chunk)
{
    // Cached per device and chunk size (multiples of 16 up to kMaxChunk).
    static int cache_all[kMaxDevices][DecodeTile<T>::kMaxChunk / 16 + 1];
    int* cache = cache_all[cur_dev()];
    const int i = chunk / 16;
    if (!cache[i]) {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_split_kernel<T, DecodeNoInline>, kDecThreads,
                                                          decode_smem_bytes<T>(chunk)) != cudaSuccess ||
            n <= 0)
            n = 1;
        cache[i] = n;
    }
    return cache[i];
}

template <typename T>
static bool set_smem_attr()
{
    static bool done[kMaxDevices];
    const int dev = cur_dev();
    if (!done[dev]) {
        const int bytes = (int)decode_smem_bytes<T>(DecodeTile<T>::kMaxChunk);
        if (cudaFuncSetAttribute(decode_split_kernel<T, DecodeNoInline>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 bytes) != cudaSuccess ||
            cudaFuncSetAttribute(decode_split_kernel<T, DecodeInline>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 bytes) != cudaSuccess ||
            cudaFuncSetAttribute(decode_split_kernel<T, DecodeInlineRow>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 bytes) != cudaSuccess)
            return false;
        done[dev] = true;
    }
    return true;
}

// Smallest chunk (multiple of 16) whose grid fits in HALF of the resident CTA slots, so
// the grid is one wave and the next kernel in the stream (launched early by programmatic
// dependent launch) finds room to start streaming its own rows meanwhile.  The largest
// chunk when none fits (then the grid runs in several waves, e.g. for large batches).
template <typename T>
static void plan(int batch, int max_kv_len, int* chunk_rows, int* nsplit, int nkvh = kHkv)
{
    set_smem_attr<T>();
    const long long slots_sms = num_sms();
    int chosen = DecodeTile<T>::kMaxChunk;
    for (int c = 16; c <= DecodeTile<T>::kMaxChunk; c += 16) {
        const long long ctas = (long long)((max_kv_len + c - 1) / c) * nkvh * batch;
        const int half_slots = blocks_per_sm<T>(c) / 2 > 0 ? blocks_per_sm<T>(c) / 2 : 1;
        if (ctas <= slots_sms * half_slots) {
            chosen = c;
            break;
        }
    }
    *chunk_rows = chosen;
    *nsplit = max_kv_len > 0 ? (max_kv_len + chosen - 1) / chosen : 0;
}

template <typename T>
static int launch_decode(const DecodeArgs& a, int batch, int nkvh, const void* inl, bool inl_row, void* stream)
{
    if (!set_smem_attr<T>()) return (int)cudaGetLastError();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.nsplit_max, nkvh, batch);
    cfg.blockDim = dim3(kDecThreads);
    cfg.dynamicSmemBytes = decode_smem_bytes<T>(a.chunk);
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (inl) {  // the parameter block is read from the host slot by the launch itself
        void* args[2] = {const_cast<DecodeArgs*>(&a), const_cast<void*>(inl)};
        return (int)cudaLaunchKernelExC(&cfg,
                                        inl_row ? (const void*)decode_split_kernel<T, DecodeInlineRow>
                                                : (const void*)decode_split_kernel<T, DecodeInline>,
                                        args);
    }
    return (int)cudaLaunchKernelEx(&cfg, decode_split_kernel<T, DecodeNoInline>, a, DecodeNoInline{});
}

// Tensor maps of a layer's K and V slabs (all row_capacity rows, boxes of `chunk` rows), kept in
// a small direct-mapped table: they depend only on the slab, so a decode step reuses the maps of
// the previous one instead of encoding two per launch (a few microseconds of host time each).
struct SlabMaps {
    CUtensorMap mk, mv;      // boxes of `chunk` rows
    CUtensorMap mk16, mv16;  // boxes of 16 rows (the last split of a sequence)
    const void* k;
    const void* v;
    int row_capacity;
    int chunk;
};
constexpr int kSlabMapSlots = 1024;
static std::mutex g_maps_mu;
static SlabMaps g_maps[kSlabMapSlots];

static bool slab_maps(const tyb_seq_kv& one, int chunk, CUtensorMap* mk, CUtensorMap* mv,
                      CUtensorMap* mk16 = nullptr, CUtensorMap* mv16 = nullptr)
{
    const uintptr_t key = reinterpret_cast<uintptr_t>(one.k);
    const size_t i = (size_t)(((key >> 8) ^ (key >> 20) ^ (uintptr_t)chunk * 0x9e37u) % kSlabMapSlots);
    std::lock_guard<std::mutex> lock(g_maps_mu);
    SlabMaps& e = g_maps[i];
    if (e.k != one.k || e.v != one.v || e.row_capacity != one.row_capacity || e.chunk != chunk) {
        if (tyb_encode_rows_map(&e.mk, one.k, one.row_capacity, one.row_capacity, chunk) != 0 ||
            tyb_encode_rows_map(&e.mv, one.v, one.row_capacity, one.row_capacity, chunk) != 0 ||
            tyb_encode_rows_map(&e.mk16, one.k, one.row_capacity, one.row_capacity, 16) != 0 ||
            tyb_encode_rows_map(&e.mv16, one.v, one.row_capacity, one.row_capacity, 16) != 0) {
            e.k = e.v = nullptr;
            return false;
        }
        e.k = one.k;
        e.v = one.v;
        e.row_capacity = one.row_capacity;
        e.chunk = chunk;
    }
    *mk = e.mk;
    *mv = e.mv;
    if (mk16) *mk16 = e.mk16;
    if (mv16) *mv16 = e.mv16;
    return true;
}

// Splits of the tensor-core form.  One sequence that fits in one CTA per SM (at most 256 rows per
// split): the split size (a multiple of 16 rows) that minimises the rows one SM must stream --
// ceil(CTAs / SMs) x rows per split, since the tile reads from shared memory bound a split and
// CTAs that share an SM share that bandwidth -- plus a fixed cost, in row equivalents, for the
// ticket and merge when there is more than one split.  At 4K context this gives 18 splits per KV
// head (144 CTAs, one per SM).  Longer sequences and request batches run in many waves: 192 rows,
// two CTAs per SM (one streams while the other computes; larger splits amortise fixed costs).
static void plan_mma(int batch, int max_kv_len, int nkvh, int* chunk_rows, int* nsplit)
{
    int best = kMmaBatchChunk;
    const long long sms = num_sms();
    if (batch == 1 && (long long)((max_kv_len + kMmaMaxChunk - 1) / kMmaMaxChunk) * nkvh <= sms) {
        long long best_cost = -1;
        for (int c = 16; c <= kMmaMaxChunk; c += 16) {
            const long long splits = (max_kv_len + c - 1) / c;
            const long long rounds = (splits * nkvh + sms - 1) / sms;
            const long long cost = rounds * c + (splits > 1 ? 300 + 4 * splits : 0);
            if (best_cost < 0 || cost <= best_cost) {
                best_cost = cost;
                best = c;
            }
        }
    }
    *chunk_rows = best;
    *nsplit = max_kv_len > 0 ? (max_kv_len + best - 1) / best : 0;
}

// Spans of the streaming form: one sequence -- as many spans as fill two CTAs per SM once,
// rounded down to whole merge batches of 32 records (32K, 8 KV heads: 725 us/step against 754
// with 37 spans); request batches -- 768 rows (8 stages).
static void plan_stream(int batch, int max_kv_len, int nkvh, int* span_rows, int* nspan)
{
    int rows = 8 * kStRows;
    if (batch == 1) {
        long long per_head = 2LL * num_sms() / nkvh;
        if (per_head >= 32) per_head -= per_head % 32;  // whole merge batches of 32 records
        if (per_head < 1) per_head = 1;
        rows = (int)(((max_kv_len + per_head - 1) / per_head + kStRows - 1) / kStRows * kStRows);
        if (rows < kStRows) rows = kStRows;
    }
    *span_rows = rows;
    *nspan = max_kv_len > 0 ? (max_kv_len + rows - 1) / rows : 0;
}

// One sequence whose splits fit in one wave at one CTA per SM takes decode_mma_kernel; longer ones
// and request batches take decode_stream_kernel.
static bool one_wave(int batch, int max_kv_len, int nkvh)
{
    return batch == 1 && (long long)((max_kv_len + kMmaMaxChunk - 1) / kMmaMaxChunk) * nkvh <= num_sms();
}

static int set_mma_smem_attr()
{
    static bool done[kMaxDevices];
    const int dev = cur_dev();
    if (!done[dev]) {
        const int mma_smem = (int)decode_mma_smem_bytes(kMmaMaxChunk), st_smem = (int)decode_stream_smem_bytes();
        const cudaFuncAttribute dyn = cudaFuncAttributeMaxDynamicSharedMemorySize;
        cudaError_t e = cudaFuncSetAttribute(decode_mma_kernel<8, false, DecodeNoInline>, dyn, mma_smem);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(decode_mma_kernel<8, true, DecodeNoInline>, dyn, mma_smem);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(decode_mma_kernel<8, false, DecodeInline>, dyn, mma_smem);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(decode_mma_kernel<8, false, DecodeInlineRow>, dyn, mma_smem);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(decode_stream_kernel<false, DecodeNoInline>, dyn, st_smem);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(decode_stream_kernel<true, DecodeNoInline>, dyn, st_smem);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(decode_stream_kernel<false, DecodeInline>, dyn, st_smem);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(decode_stream_kernel<false, DecodeInlineRow>, dyn, st_smem);
        if (e != cudaSuccess) return (int)e;
        done[dev] = true;
    }
    return 0;
}

// The tensor-core form for one sequence with a BF16 cache.  Splits as planned for
// decode_split_kernel<bf16> (same record count, so the callers' workspaces fit).
static int launch_decode_mma(DecodeMmaArgs a, const tyb_seq_kv& one, int nkvh, const void* inl, bool inl_row,
                             void* stream)
{
    const int e = set_mma_smem_attr();
    if (e) return e;
    CUtensorMap mk, mv, mk16, mv16;
    if (!slab_maps(one, a.chunk, &mk, &mv, &mk16, &mv16)) return (int)cudaErrorInvalidValue;
    a.seqs = nullptr;
    a.maps = nullptr;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.nsplit, nkvh, 1);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = decode_mma_smem_bytes(a.chunk);
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (inl) {  // the parameter block is read from the host slot by the launch itself
        if (a.q_norm) return (int)cudaErrorInvalidValue;
        void* args[6] = {&mk, &mv, &mk16, &mv16, &a, const_cast<void*>(inl)};
        return (int)cudaLaunchKernelExC(&cfg,
                                        inl_row ? (const void*)decode_mma_kernel<8, false, DecodeInlineRow>
                                                : (const void*)decode_mma_kernel<8, false, DecodeInline>,
                                        args);
    }
    if (a.q_norm)
        return (int)cudaLaunchKernelEx(&cfg, decode_mma_kernel<8, true, DecodeNoInline>, mk, mv, mk16, mv16, a,
                                       DecodeNoInline{});
    return (int)cudaLaunchKernelEx(&cfg, decode_mma_kernel<8, false, DecodeNoInline>, mk, mv, mk16, mv16, a,
                                   DecodeNoInline{});
}

static int launch_stream(const DecodeMmaArgs& a, const CUtensorMap& mk, const CUtensorMap& mv, int nkvh, int batch,
                         const void* inl, bool inl_row, void* stream)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.nsplit, nkvh, batch);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = decode_stream_smem_bytes();
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (inl) {
        if (a.q_norm) return (int)cudaErrorInvalidValue;
        void* args[4] = {const_cast<CUtensorMap*>(&mk), const_cast<CUtensorMap*>(&mv), const_cast<DecodeMmaArgs*>(&a),
                         const_cast<void*>(inl)};
        return (int)cudaLaunchKernelExC(&cfg,
                                        inl_row ? (const void*)decode_stream_kernel<false, DecodeInlineRow>
                                                : (const void*)decode_stream_kernel<false, DecodeInline>,
                                        args);
    }
    if (a.q_norm) return (int)cudaLaunchKernelEx(&cfg, decode_stream_kernel<true, DecodeNoInline>, mk, mv, a, DecodeNoInline{});
    return (int)cudaLaunchKernelEx(&cfg, decode_stream_kernel<false, DecodeNoInline>, mk, mv, a, DecodeNoInline{});
}

}  // namespace tyb

using namespace tyb;

extern "C" size_t tyb_decode_maps_bytes(int batch) { return (size_t)batch * 2 * sizeof(CUtensorMap); }

extern "C" int tyb_decode_launch_batched(const float* q, float* out, const tyb_seq_kv* seqs_host, void* upload,
                                         int batch, int max_kv_len, float scale, float* partials,
                                         unsigned int* counters, void* stream)
{
    if (batch <= 0 || max_kv_len <= 0) return 0;
    int e = set_mma_smem_attr();
    if (e) return e;
    int chunk, nsplit;
    plan_stream(batch, max_kv_len, kHkv, &chunk, &nsplit);
    // Host staging: [maps 2 x batch][descriptors batch], one pageable copy (staged by the driver
    // before cudaMemcpyAsync returns, so the buffer may be freed right after).
    const size_t maps_bytes = tyb_decode_maps_bytes(batch);
    const size_t bytes = maps_bytes + sizeof(tyb_seq_kv) * (size_t)batch;
    CUtensorMap* host = static_cast<CUtensorMap*>(aligned_alloc(64, (bytes + 63) & ~size_t(63)));
    if (!host) return (int)cudaErrorMemoryAllocation;
    for (int b = 0; b < batch; b++) {
        if (!slab_maps(seqs_host[b], kStRows, &host[2 * b], &host[2 * b + 1])) {
            free(host);
            return (int)cudaErrorInvalidValue;
        }
    }
    memcpy(reinterpret_cast<unsigned char*>(host) + maps_bytes, seqs_host, sizeof(tyb_seq_kv) * (size_t)batch);
    cudaError_t ce = cudaMemcpyAsync(upload, host, bytes, cudaMemcpyHostToDevice, (cudaStream_t)stream);
    const CUtensorMap m0 = host[0], m1 = host[1];
    free(host);
    if (ce != cudaSuccess) return (int)ce;
    DecodeMmaArgs a = {};
    a.q = q;
    a.out = out;
    a.seqs = reinterpret_cast<const tyb_seq_kv*>(static_cast<unsigned char*>(upload) + maps_bytes);
    a.maps = static_cast<const CUtensorMap*>(upload);
    a.scale_log2 = scale * kLog2e;
    a.chunk = chunk;    // rows per span
    a.nsplit = nsplit;  // the record stride; each sequence's own span count comes from its length
    a.partials = partials;
    a.counters = counters;
    a.prefetch_small = 1;
    a.gather = nullptr;
    return launch_stream(a, m0, m1, kHkv, batch, nullptr, false, stream);
}

extern "C" void tyb_decode_plan(int batch, int max_kv_len, int kv_dtype, int* chunk_rows, int* nsplit)
{
    if (kv_dtype == TYB_BF16 && one_wave(batch, max_kv_len, kHkv))
        plan_mma(batch, max_kv_len, kHkv, chunk_rows, nsplit);
    else if (kv_dtype == TYB_BF16)
        plan_stream(batch, max_kv_len, kHkv, chunk_rows, nsplit);  // spans
    else
        plan<float>(batch, max_kv_len, chunk_rows, nsplit);
}

extern "C" size_t tyb_decode_partial_floats(int batch, int nsplit)
{
    return (size_t)batch * kHkv * (size_t)nsplit * kRec;
}

static int launch_heads_impl(const float* q, float* out, const tyb_seq_kv* seqs_dev, tyb_seq_kv one, int batch,
                             int max_kv_len, int kv_dtype, float scale, float* partials, unsigned int* counters,
                             const float* k_new, const float* v_new, int prefetch_rows, int kvh0, int nkvh,
                             int flags, const void* gather, const tyb_qk_prep* prep, const float* inl, void* stream)
{
    if (gather && (kv_dtype != TYB_BF16 || seqs_dev || batch != 1)) return (int)cudaErrorInvalidValue;
    // Inputs in the parameter block: one sequence, no gather, raw-pointer decode (not the QK-norm form)
    if (inl && (seqs_dev || batch != 1 || gather || prep)) return (int)cudaErrorInvalidValue;
    if (inl) flags &= ~TYB_DEC_DEVICE_SMALL;
    const bool inl_row = (flags & TYB_DEC_INLINE_ROW) != 0;
    // QK-RMSNorm + M-RoPE on load: the tensor-core forms for one sequence (BF16 cache) only
    if (prep && (kv_dtype != TYB_BF16 || seqs_dev || batch != 1 || !prep->q_norm || !prep->k_norm ||
                 !prep->cos || !prep->sin))
        return (int)cudaErrorInvalidValue;
    if (batch <= 0 || max_kv_len <= 0 || nkvh <= 0) return 0;
    DecodeArgs a;
    a.kvh0 = kvh0;
    a.prefetch_small = (flags & TYB_DEC_DEVICE_SMALL) != 0;
    a.q = q;
    a.out = out;
    a.seqs = seqs_dev;
    a.one = one;
    a.k_new = k_new;
    a.v_new = v_new;
    a.scale_log2 = scale * kLog2e;
    int chunk, nsplit;
    const bool bf16_one = kv_dtype == TYB_BF16 && !seqs_dev && batch == 1;
    if (bf16_one && one_wave(1, max_kv_len, nkvh))
        plan_mma(1, max_kv_len, nkvh, &chunk, &nsplit);
    else if (bf16_one)
        plan_stream(1, max_kv_len, nkvh, &chunk, &nsplit);
    else if (kv_dtype == TYB_BF16)
        plan<__nv_bfloat16>(batch, max_kv_len, &chunk, &nsplit, nkvh);
    else
        plan<float>(batch, max_kv_len, &chunk, &nsplit, nkvh);
    a.chunk = chunk;
    a.nsplit_max = nsplit;
    a.prefetch_rows = seqs_dev ? 0 : prefetch_rows;
    a.partials = partials;
    a.counters = counters;
    if (bf16_one) {
        DecodeMmaArgs m = {};
        m.q = q;
        m.out = out;
        m.k = static_cast<__nv_bfloat16*>(const_cast<void*>(one.k));
        m.v = static_cast<__nv_bfloat16*>(const_cast<void*>(one.v));
        m.row_capacity = one.row_capacity;
        m.kv_len = one.kv_len;
        m.k_new = k_new;
        m.v_new = v_new;
        m.scale_log2 = a.scale_log2;
        m.chunk = chunk;
        m.nsplit = (one.kv_len + chunk - 1) / chunk;
        m.prefetch_rows = prefetch_rows;
        m.partials = partials;
        m.counters = counters;
        m.kvh0 = kvh0;
        m.prefetch_small = a.prefetch_small;
        m.wide_counters = (flags & TYB_DEC_WIDE_COUNTERS) != 0;
        m.gather = static_cast<const GatherDev*>(gather);
        if (prep) {
            m.q_norm = prep->q_norm;
            m.k_norm = prep->k_norm;
            m.rope_cos = prep->cos;
            m.rope_sin = prep->sin;
            m.eps = prep->eps;
        }
        if (one_wave(1, max_kv_len, nkvh)) return launch_decode_mma(m, one, nkvh, inl, inl_row, stream);
        const int e = set_mma_smem_attr();
        if (e) return e;
        CUtensorMap mk, mv;
        if (!slab_maps(one, kStRows, &mk, &mv)) return (int)cudaErrorInvalidValue;
        m.seqs = nullptr;
        m.maps = nullptr;
        return launch_stream(m, mk, mv, nkvh, 1, inl, inl_row, stream);
    }
    if (kv_dtype == TYB_BF16) return launch_decode<__nv_bfloat16>(a, batch, nkvh, inl, inl_row, stream);
    return launch_decode<float>(a, batch, nkvh, inl, inl_row, stream);
}

extern "C" int tyb_decode_launch_heads(const float* q, float* out, const tyb_seq_kv* seqs_dev, tyb_seq_kv one,
                                       int batch, int max_kv_len, int kv_dtype, float scale, float* partials,
                                       unsigned int* counters, const float* k_new, const float* v_new,
                                       int prefetch_rows, int kvh0, int nkvh, int flags, const void* gather,
                                       const float* inl, void* stream)
{
    return launch_heads_impl(q, out, seqs_dev, one, batch, max_kv_len, kv_dtype, scale, partials, counters, k_new,
                             v_new, prefetch_rows, kvh0, nkvh, flags, gather, nullptr, inl, stream);
}

extern "C" int tyb_decode_launch_fused(const float* q_raw, float* out, tyb_seq_kv one, int kv_len, float scale,
                                       float* partials, unsigned int* counters, const float* k_raw,
                                       const float* v_new, int prefetch_rows, const tyb_qk_prep* prep, void* stream)
{
    if (!prep) return (int)cudaErrorInvalidValue;
    return launch_heads_impl(q_raw, out, nullptr, one, 1, kv_len, TYB_BF16, scale, partials, counters, k_raw, v_new,
                             prefetch_rows, 0, kHkv, TYB_DEC_DEVICE_SMALL | TYB_DEC_WIDE_COUNTERS, nullptr, prep,
                             nullptr, stream);
}

extern "C" int tyb_decode_launch_ex(const float* q, float* out, const tyb_seq_kv* seqs_dev, tyb_seq_kv one,
                                    int batch, int max_kv_len, int kv_dtype, float scale, float* partials,
                                    unsigned int* counters, const float* k_new, const float* v_new,
                                    int prefetch_rows, void* stream)
{
    return tyb_decode_launch_heads(q, out, seqs_dev, one, batch, max_kv_len, kv_dtype, scale, partials, counters,
                                   k_new, v_new, prefetch_rows, 0, kHkv, 0, nullptr, nullptr, stream);
}

extern "C" int tyb_decode_launch(const float* q, float* out, const tyb_seq_kv* seqs_dev, tyb_seq_kv one,
                                 int batch, int max_kv_len, int kv_dtype, float scale, float* partials,
                                 unsigned int* counters, void* stream)
{
    return tyb_decode_launch_ex(q, out, seqs_dev, one, batch, max_kv_len, kv_dtype, scale, partials, counters,
                                nullptr, nullptr, 0, stream);
}

// ---- decode that allocates nothing ----------------------------------------------------------
//
// Some callers cannot call cudaMalloc: a serving engine whose device memory is all reserved
// up front by its own caching allocator (an allocation behind its back can fail or fragment
// that pool), or a host program that keeps a fixed, audited device-memory footprint.  For
// them this entry point runs the same split-KV kernel with its split records and tickets in
// a fixed file-scope device array instead of a cache's workspace.  The array (about 2 MiB)
// exists on every GPU that loads this library until the process exits.

namespace tyb {

constexpr int kNoAllocMaxSplits = 256;
constexpr int kNoAllocMaxDevices = 64;
static __device__ __align__(256) float g_noalloc_records[kHkv * kNoAllocMaxSplits * kRec];
static __device__ __align__(256) unsigned int g_noalloc_tickets[kHkv];

// Device addresses of the two arrays, looked up once per device.  In host code the
// arrays' names only stand in for the device symbols; kernels must get these addresses.
static std::mutex g_noalloc_mu;
static float* g_noalloc_records_addr[kNoAllocMaxDevices];
static unsigned int* g_noalloc_tickets_addr[kNoAllocMaxDevices];

static bool is_device_memory(const void* p)
{
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged;
}

}  // namespace tyb

extern "C" int attention_decode_gqa_noalloc(const float* q, const void* k_rows, const void* v_rows,
                                            int row_capacity, int kv_dtype, float* output, int kv_len,
                                            float scale, void* stream)
{
    const char* what = "attention_decode_gqa_noalloc";
    if (!q || !k_rows || !v_rows || !output) {
        tyb_set_error("%s: NULL q/k_rows/v_rows/output", what);
        return 1;
    }
    if (kv_dtype != TYB_F32 && kv_dtype != TYB_BF16) {
        tyb_set_error("%s: unknown kv_dtype %d", what, kv_dtype);
        return 1;
    }
    if (row_capacity <= 0 || kv_len < 1 || kv_len > row_capacity) {
        tyb_set_error("%s: need 1 <= kv_len (%d) <= row_capacity (%d)", what, kv_len, row_capacity);
        return 1;
    }
    if ((reinterpret_cast<uintptr_t>(k_rows) | reinterpret_cast<uintptr_t>(v_rows)) & 15u) {
        tyb_set_error("%s: k_rows and v_rows must be 16-byte aligned", what);
        return 1;
    }
    // The kernels read the query and write the output with 16-byte vector accesses.
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(output)) & 15u) {
        tyb_set_error("%s: q and output must be 16-byte aligned", what);
        return 1;
    }
    if (!is_device_memory(q) || !is_device_memory(k_rows) || !is_device_memory(v_rows) ||
        !is_device_memory(output)) {
        tyb_set_error("%s: q, k_rows, v_rows and output must be device memory", what);
        return 1;
    }
    int chunk = 0, nsplit = 0;
    tyb_decode_plan(1, kv_len, kv_dtype, &chunk, &nsplit);
    if (nsplit > kNoAllocMaxSplits) {
        const int max_chunk = DecodeTile<float>::kMaxChunk;  // BF16 never gets here (at most 2 x SMs / 8 spans)
        tyb_set_error("%s: kv_len %d needs %d splits; the fixed scratch holds %d (kv_len <= %d for this "
                      "element type)",
                      what, kv_len, nsplit, kNoAllocMaxSplits, kNoAllocMaxSplits * max_chunk);
        return 1;
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) {
        tyb_set_error("%s: no usable current device (%s)", what, cudaGetErrorString(e));
        return 1;
    }
    float* records = nullptr;
    unsigned int* tickets = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        if (!g_noalloc_records_addr[dev]) {
            void* r = nullptr;
            void* t = nullptr;
            e = cudaGetSymbolAddress(&r, g_noalloc_records);
            if (e == cudaSuccess) e = cudaGetSymbolAddress(&t, g_noalloc_tickets);
            if (e != cudaSuccess) {
                tyb_set_error("%s: cudaGetSymbolAddress: %s", what, cudaGetErrorString(e));
                return 1;
            }
            g_noalloc_records_addr[dev] = static_cast<float*>(r);
            g_noalloc_tickets_addr[dev] = static_cast<unsigned int*>(t);
        }
        records = g_noalloc_records_addr[dev];
        tickets = g_noalloc_tickets_addr[dev];
    }
    // The array keeps the previous call's contents: tickets must start at zero.
    e = cudaMemsetAsync(tickets, 0, sizeof(unsigned int) * kHkv, (cudaStream_t)stream);
    if (e != cudaSuccess) {
        tyb_set_error("%s: cudaMemsetAsync: %s", what, cudaGetErrorString(e));
        return 1;
    }
    tyb_seq_kv one;
    one.k = k_rows;
    one.v = v_rows;
    one.kv_len = kv_len;
    one.row_capacity = row_capacity;
    one.pf_k = one.pf_v = nullptr;
    const int rc = tyb_decode_launch(q, output, nullptr, one, 1, kv_len, kv_dtype, scale, records, tickets, stream);
    if (rc != 0) {
        tyb_set_error("%s: launch: %s", what, cudaGetErrorString((cudaError_t)rc));
        return 1;
    }
    return 0;
}

// ---- decode output gather: host side ----------------------------------------------------------

namespace tyb {

struct GatherHost {
    GatherBuf* local = nullptr;  // this rank's exchange buffer
    GatherDev* dev = nullptr;    // device table
    GatherBuf* peer[kGatherMaxRanks] = {};
    int rank = -1;
    int world = 0;
    bool connected = false;
};
static GatherHost g_gather;
static std::mutex g_gather_mu;

}  // namespace tyb

extern "C" int tyb_gather_init(int rank, int world)
{
    std::lock_guard<std::mutex> lock(g_gather_mu);
    if (world < 1 || world > kGatherMaxRanks || rank < 0 || rank >= world) return (int)cudaErrorInvalidValue;
    if (g_gather.local) return (int)cudaErrorInvalidValue;  // already set up: close first
    cudaError_t e = cudaMalloc(&g_gather.local, sizeof(GatherBuf));
    if (e == cudaSuccess) e = cudaMemset(g_gather.local, 0, sizeof(GatherBuf));
    if (e == cudaSuccess) e = cudaMalloc(&g_gather.dev, sizeof(GatherDev));
    if (e != cudaSuccess) {
        cudaFree(g_gather.local);
        g_gather.local = nullptr;
        return (int)e;
    }
    g_gather.rank = rank;
    g_gather.world = world;
    return 0;
}

extern "C" int tyb_gather_handle(void* handle_out)
{
    if (!g_gather.local || !handle_out) return (int)cudaErrorInvalidValue;
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, g_gather.local);
    if (e != cudaSuccess) return (int)e;
    memcpy(handle_out, &h, sizeof h);
    return 0;
}

extern "C" int tyb_gather_connect(const void* handles)
{
    std::lock_guard<std::mutex> lock(g_gather_mu);
    if (!g_gather.local || !handles || g_gather.connected) return (int)cudaErrorInvalidValue;
    GatherDev d = {};
    d.rank = g_gather.rank;
    d.world = g_gather.world;
    for (int p = 0; p < g_gather.world; p++) {
        if (p == g_gather.rank) {
            d.buf[p] = g_gather.local;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const unsigned char*>(handles) + (size_t)p * sizeof h, sizeof h);
        void* ptr = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (int q = 0; q < p; q++)
                if (g_gather.peer[q]) cudaIpcCloseMemHandle(g_gather.peer[q]);
            return (int)e;
        }
        g_gather.peer[p] = static_cast<GatherBuf*>(ptr);
        d.buf[p] = g_gather.peer[p];
    }
    const cudaError_t e = cudaMemcpy(g_gather.dev, &d, sizeof d, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return (int)e;
    g_gather.connected = true;
    return 0;
}

extern "C" const void* tyb_gather_dev(int* world, int* rank)
{
    if (!g_gather.connected) return nullptr;
    if (world) *world = g_gather.world;
    if (rank) *rank = g_gather.rank;
    return g_gather.dev;
}

extern "C" void tyb_gather_close(void)
{
    std::lock_guard<std::mutex> lock(g_gather_mu);
    cudaDeviceSynchronize();
    for (int p = 0; p < kGatherMaxRanks; p++) {
        if (g_gather.peer[p]) cudaIpcCloseMemHandle(g_gather.peer[p]);
        g_gather.peer[p] = nullptr;
    }
    cudaFree(g_gather.dev);
    cudaFree(g_gather.local);
    g_gather = GatherHost();
}
