// decode.cu -- split-KV flash decoding for one new token per sequence, optionally fused
// with the KV append of that token.
//
// Replaces the reference's per-KV-head CPU worker (kernel/attention.c:158-204: for each
// KV head and its two query heads, scores = q.K*scale over kv_len rows, max, exp, sum,
// normalise, out = sum p*V) and, fused, kernel/kv_cache.c:53-65 (the new row written at
// row seq_len first).  One CTA owns one (sequence, KV head, split of rows):
//   1. one thread starts two bulk async copies (TMA, 1-D) of the split's K and V rows --
//      contiguous in the head-first cache -- into shared memory on two mbarriers.  The
//      kernel is launched with programmatic dependent launch and the grid is planned to
//      fill only half of the SM slots, so the next kernel's CTAs are resident early and
//      request their rows BEFORE griddepcontrol.wait (only rows the host knows the
//      previous launch did not write); the stream of K/V bytes continues across kernels;
//   2. after the wait: the query (and the new row, written to the cache and into its
//      slot), scores of both query heads (16-byte vectors, 16 lanes per row, shuffle-xor
//      reduction), max and exp2 per head;
//   3. p.V for both heads from the same V bytes (GQA pair read once);
//   4. the split's (max, sum, unnormalised o) goes to a workspace record; the CTA that
//      takes the last ticket merges all records, pulled into shared memory by bulk
//      copies, and writes the output.  No second launch.
// Bandwidth-bound: 2 * kv_len * 128 * sizeof(T) bytes per (sequence, KV head).
#include <mutex>

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
};

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
// [V (reused for merge weights)] [scores 2 x chunk] [stat 24] [2 mbarriers] [flag].
template <typename T>
__host__ __device__ constexpr size_t dec_k_region(int chunk)
{
    return dec_kv_bytes<T>(chunk) > (size_t)kRedBytes ? dec_kv_bytes<T>(chunk) : (size_t)kRedBytes;
}

template <typename T>
__host__ __device__ constexpr size_t decode_smem_bytes(int chunk)
{
    return dec_k_region<T>(chunk) + dec_kv_bytes<T>(chunk) + sizeof(float) * (2 * chunk + 24) + 2 * sizeof(uint64_t) +
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

template <typename T>
__global__ void __launch_bounds__(kDecThreads, 2) decode_split_kernel(const DecodeArgs a)
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
    uint64_t* bars = reinterpret_cast<uint64_t*>(stat + 24);
    int* last_flag = reinterpret_cast<int*>(bars + 2);
    float* red = reinterpret_cast<float*>(kreg);  // [16][2][128], after the scores

    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        fence_barrier_init();
        fence_proxy_async_smem();
    }
    __syncthreads();

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
    // requested before waiting for the previous kernel when that kernel did not write them.
    bool issued = false;
    if (!a.seqs) {
        geometry(a.one);
        if (tid == 0 && s < nsplit && r0 + tma_rows <= a.prefetch_rows) {
            issue();
            issued = true;
        }
    }
    // Everything below reads data earlier kernels wrote (descriptors, cache rows, q).
    pdl_wait();
    pdl_trigger();
    if (a.seqs) geometry(a.seqs[b]);
    if (s >= nsplit) return;
    if (tid == 0 && !issued) issue();

    // Query vectors of the two heads sharing this KV head, for the scores: 8 lanes per row,
    // lane part p holds the 16 dims of load_lane16.
    const int g16 = lane & 15;
    const int part = lane & 7;
    float q0[16], q1[16];
    {
        const float* qb = a.q + (size_t)b * kHq * kD + (size_t)(kGroup * kvh) * kD;
        load_query16<T>(qb, part, q0);
        load_query16<T>(qb + kD, part, q1);
    }

    // The new token's row (fused append): threads 0..15 write it to the cache and into its
    // slot after the copied rows (K now, V once V has landed).
    const bool has_new = a.k_new && kv_len - 1 >= r0 && kv_len - 1 < r0 + nrows;
    float nk[8], nv[8];
    if (has_new && tid < 16) {
        const size_t off = ((size_t)b * kHkv + kvh) * kD + tid * 8;
        load8(a.k_new + off, nk);
        load8(a.v_new + off, nv);
        store8(const_cast<T*>(kh) + (size_t)(kv_len - 1) * kD + tid * 8, nk);
        store8(const_cast<T*>(vh) + (size_t)(kv_len - 1) * kD + tid * 8, nv);
        store8(Ks + (size_t)(kv_len - 1 - r0) * kD + tid * 8, nk);
    }

    // Every thread waits (bounded); the CTA leaves together if any wait ran out.
    if (__syncthreads_or(!mbar_wait_bounded(&bars[0], 0, kWaitLimitNs, TYB_STATUS_WAIT_TIMEOUT))) return;

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
    if (__syncthreads_or(!mbar_wait_bounded(&bars[1], 0, kWaitLimitNs, TYB_STATUS_WAIT_TIMEOUT))) return;

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
    // Records arrive in shared memory in batches by one bulk copy each; every thread then
    // merges one output element (h, d) from shared memory, with an online max across batches.
    float* region = reinterpret_cast<float*>(kreg);  // K and V regions are free now
    const size_t region_bytes = dec_k_region<T>(a.chunk) + dec_kv_bytes<T>(a.chunk);
    const int cap = (int)(region_bytes / (sizeof(float) * (kRec + 2)));
    float* wts = region + (size_t)cap * kRec;  // [cap][2]
    float run0 = -INFINITY, run1 = -INFINITY;  // running max of each head (uniform)
    float L = 0.f, O = 0.f;                     // this thread's head h, element d
    uint32_t phase = 1;                         // bars[0] completed phase 0 with the K rows
    for (int j0 = 0; j0 < nsplit; j0 += cap) {
        const int nb = min(cap, nsplit - j0);
        __syncthreads();  // the previous batch is consumed
        if (tid == 0) {
            const uint32_t bytes = (uint32_t)nb * kRec * sizeof(float);
            mbar_arrive_expect_tx(&bars[0], bytes);
            bulk_g2s(region, recs + (size_t)j0 * kRec, bytes, &bars[0]);
        }
        if (__syncthreads_or(!mbar_wait_bounded(&bars[0], phase, kWaitLimitNs, TYB_STATUS_WAIT_TIMEOUT))) return;
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
            sc[warp] = x0;
            sc[16 + warp] = x1;
        }
        __syncthreads();
        float n0 = run0, n1 = run1;
#pragma unroll
        for (int w = 0; w < kDecThreads / 32; w++) {
            n0 = fmaxf(n0, sc[w]);
            n1 = fmaxf(n1, sc[16 + w]);
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
    a.out[out_head + (size_t)h * kD + d] = O / L;
    if (tid == 0) a.counters[b * kHkv + kvh] = 0u;
}

// ---- host-side planning ----------------------------------------------------------------

static int g_num_sms = 0;

static int num_sms()
{
    if (!g_num_sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || g_num_sms <= 0)
            g_num_sms = 148;
    }
    return g_num_sms;
}

template <typename T>
static int blocks_per_sm(int chunk)
{
    // Cached per chunk size (multiples of 16 up to kMaxChunk).
    static int cache[DecodeTile<T>::kMaxChunk / 16 + 1];
    const int i = chunk / 16;
    if (!cache[i]) {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_split_kernel<T>, kDecThreads,
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
    static bool done = false;
    if (!done) {
        if (cudaFuncSetAttribute(decode_split_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)decode_smem_bytes<T>(DecodeTile<T>::kMaxChunk)) != cudaSuccess)
            return false;
        done = true;
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
static int launch_decode(const DecodeArgs& a, int batch, int nkvh, void* stream)
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
    return (int)cudaLaunchKernelEx(&cfg, decode_split_kernel<T>, a);
}

}  // namespace tyb

using namespace tyb;

extern "C" void tyb_decode_plan(int batch, int max_kv_len, int kv_dtype, int* chunk_rows, int* nsplit)
{
    if (kv_dtype == TYB_BF16)
        plan<__nv_bfloat16>(batch, max_kv_len, chunk_rows, nsplit);
    else
        plan<float>(batch, max_kv_len, chunk_rows, nsplit);
}

extern "C" size_t tyb_decode_partial_floats(int batch, int nsplit)
{
    return (size_t)batch * kHkv * (size_t)nsplit * kRec;
}

extern "C" int tyb_decode_launch_heads(const float* q, float* out, const tyb_seq_kv* seqs_dev, tyb_seq_kv one,
                                       int batch, int max_kv_len, int kv_dtype, float scale, float* partials,
                                       unsigned int* counters, const float* k_new, const float* v_new,
                                       int prefetch_rows, int kvh0, int nkvh, void* stream)
{
    if (batch <= 0 || max_kv_len <= 0 || nkvh <= 0) return 0;
    DecodeArgs a;
    a.kvh0 = kvh0;
    a.q = q;
    a.out = out;
    a.seqs = seqs_dev;
    a.one = one;
    a.k_new = k_new;
    a.v_new = v_new;
    a.scale_log2 = scale * kLog2e;
    int chunk, nsplit;
    if (kv_dtype == TYB_BF16)
        plan<__nv_bfloat16>(batch, max_kv_len, &chunk, &nsplit, nkvh);
    else
        plan<float>(batch, max_kv_len, &chunk, &nsplit, nkvh);
    a.chunk = chunk;
    a.nsplit_max = nsplit;
    a.prefetch_rows = seqs_dev ? 0 : prefetch_rows;
    a.partials = partials;
    a.counters = counters;
    if (kv_dtype == TYB_BF16) return launch_decode<__nv_bfloat16>(a, batch, nkvh, stream);
    return launch_decode<float>(a, batch, nkvh, stream);
}

extern "C" int tyb_decode_launch_ex(const float* q, float* out, const tyb_seq_kv* seqs_dev, tyb_seq_kv one,
                                    int batch, int max_kv_len, int kv_dtype, float scale, float* partials,
                                    unsigned int* counters, const float* k_new, const float* v_new,
                                    int prefetch_rows, void* stream)
{
    return tyb_decode_launch_heads(q, out, seqs_dev, one, batch, max_kv_len, kv_dtype, scale, partials, counters,
                                   k_new, v_new, prefetch_rows, 0, kHkv, stream);
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
    if (!is_device_memory(q) || !is_device_memory(k_rows) || !is_device_memory(v_rows) ||
        !is_device_memory(output)) {
        tyb_set_error("%s: q, k_rows, v_rows and output must be device memory", what);
        return 1;
    }
    int chunk = 0, nsplit = 0;
    tyb_decode_plan(1, kv_len, kv_dtype, &chunk, &nsplit);
    if (nsplit > kNoAllocMaxSplits) {
        const int max_chunk =
            kv_dtype == TYB_BF16 ? DecodeTile<__nv_bfloat16>::kMaxChunk : DecodeTile<float>::kMaxChunk;
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
    const int rc = tyb_decode_launch(q, output, nullptr, one, 1, kv_len, kv_dtype, scale, records, tickets, stream);
    if (rc != 0) {
        tyb_set_error("%s: launch: %s", what, cudaGetErrorString((cudaError_t)rc));
        return 1;
    }
    return 0;
}
