// decode.cu -- split-KV flash decoding for one new token per sequence.
//
// Replaces the reference's per-KV-head CPU worker (kernel/attention.c:158-204: for each
// KV head and its two query heads, scores = q.K*scale over kv_len rows, max, exp, sum,
// normalise, out = sum p*V).  Here one CTA owns one (sequence, KV head, split of rows):
//   1. one thread starts two bulk async copies (TMA, 1-D) of the split's K and V rows --
//      contiguous in the head-first cache -- into shared memory, each completing on
//      its own mbarrier, so the whole split is in flight before any math runs;
//   2. the CTA computes both query heads' scores against K (16-byte vectors, 16 lanes
//      per row, shuffle-xor reduction), then max and exp2 per head;
//   3. once V has landed, p.V for both heads (K/V read once for the GQA pair);
//   4. the split's (max, sum, unnormalised o) goes to a workspace and the last CTA of
//      the (sequence, head) -- found with an atomic ticket -- merges all splits and
//      writes the output.  No second launch.
// Bandwidth-bound: 2 * kv_len * 128 * sizeof(T) bytes per (sequence, KV head).
#include "common.cuh"

namespace tyb {

constexpr int kDecThreads = 128;
constexpr int kPartStride = 132;  // m, l, 2 pad, o[128]: keeps o 16-byte aligned

template <typename T>
struct DecodeTile {
    // Rows per split are capped so K+V of one split stay <= 64 KB of shared memory,
    // which leaves room for three CTAs per SM.
    static constexpr int kMaxChunk = 65536 / (2 * kD * (int)sizeof(T));
};

struct DecodeArgs {
    const float* q;
    float* out;
    const tyb_seq_kv* seqs;
    tyb_seq_kv one;
    float scale_log2;
    int chunk;
    int nsplit_max;
    float* partials;
    unsigned int* counters;
};

__device__ __forceinline__ float fast_exp2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <typename T>
__global__ void __launch_bounds__(kDecThreads) decode_split_kernel(const DecodeArgs a)
{
    extern __shared__ __align__(128) unsigned char smem[];
    const int s = blockIdx.x;
    const int kvh = blockIdx.y;
    const int b = blockIdx.z;
    const tyb_seq_kv seq = a.seqs ? a.seqs[b] : a.one;
    const int kv_len = seq.kv_len;
    const int nsplit = (kv_len + a.chunk - 1) / a.chunk;
    if (s >= nsplit) return;
    const int r0 = s * a.chunk;
    const int nrows = min(a.chunk, kv_len - r0);

    T* Ks = reinterpret_cast<T*>(smem);
    T* Vs = Ks + (size_t)a.chunk * kD;
    float* sc = reinterpret_cast<float*>(Vs + (size_t)a.chunk * kD);  // [2][chunk]
    float* red = sc + 2 * a.chunk;                                    // [8][2][128]
    float* stat = red + 8 * 2 * kD;                                   // m0 m1 l0 l1
    uint64_t* bars = reinterpret_cast<uint64_t*>(stat + 8);
    int* last_flag = reinterpret_cast<int*>(bars + 2);

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const size_t head_off = ((size_t)kvh * seq.row_capacity + r0) * kD;

    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        fence_barrier_init();
        fence_proxy_async_smem();
    }
    __syncthreads();
    if (tid == 0) {
        const uint32_t bytes = (uint32_t)nrows * kD * sizeof(T);
        mbar_arrive_expect_tx(&bars[0], bytes);
        bulk_g2s(Ks, static_cast<const T*>(seq.k) + head_off, bytes, &bars[0]);
        mbar_arrive_expect_tx(&bars[1], bytes);
        bulk_g2s(Vs, static_cast<const T*>(seq.v) + head_off, bytes, &bars[1]);
    }

    // Query vectors of the two heads sharing this KV head: lane group g16 holds dims
    // [8*g16, 8*g16+8).
    const int g16 = lane & 15;
    float q0[8], q1[8];
    {
        const float* qb = a.q + (size_t)b * kHq * kD + (size_t)(kGroup * kvh) * kD + g16 * 8;
        load8(qb, q0);
        load8(qb + kD, q1);
    }

    // Every thread waits (bounded); the CTA leaves together if any wait ran out.
    if (__syncthreads_or(!mbar_wait_bounded(&bars[0], 0, kWaitLimitNs, TYB_STATUS_WAIT_TIMEOUT)))
        return;

    // Scores: each warp pass covers two rows (one per 16-lane half).
    const int half = lane >> 4;
    for (int p = warp; 2 * p < nrows; p += kDecThreads / 32) {
        const int r = 2 * p + half;
        float d0 = 0.f, d1 = 0.f;
        if (r < nrows) {
            float k8[8];
            load8(Ks + (size_t)r * kD + g16 * 8, k8);
#pragma unroll
            for (int j = 0; j < 8; j++) {
                d0 = fmaf(q0[j], k8[j], d0);
                d1 = fmaf(q1[j], k8[j], d1);
            }
        }
#pragma unroll
        for (int off = 8; off >= 1; off >>= 1) {
            d0 += __shfl_xor_sync(0xffffffffu, d0, off);
            d1 += __shfl_xor_sync(0xffffffffu, d1, off);
        }
        if (g16 == 0 && r < nrows) {
            sc[r] = d0 * a.scale_log2;
            sc[a.chunk + r] = d1 * a.scale_log2;
        }
    }
    __syncthreads();

    // Max and exp2 per head: warp 0 takes head 0, warp 1 head 1.
    if (warp < 2) {
        float* row = sc + warp * a.chunk;
        float m = -INFINITY;
        for (int r = lane; r < nrows; r += 32) m = fmaxf(m, row[r]);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
        float l = 0.f;
        for (int r = lane; r < nrows; r += 32) {
            const float e = fast_exp2(row[r] - m);
            row[r] = e;
            l += e;
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
        if (lane == 0) {
            stat[warp] = m;
            stat[2 + warp] = l;
        }
    }
    __syncthreads();

    if (__syncthreads_or(!mbar_wait_bounded(&bars[1], 0, kWaitLimitNs, TYB_STATUS_WAIT_TIMEOUT)))
        return;

    // p.V: thread owns dims [8*g16, +8) of rows rg, rg+8, ...
    const int rg = tid >> 4;
    float o0[8], o1[8];
#pragma unroll
    for (int j = 0; j < 8; j++) o0[j] = o1[j] = 0.f;
    for (int r = rg; r < nrows; r += kDecThreads / 16) {
        float v8[8];
        load8(Vs + (size_t)r * kD + g16 * 8, v8);
        const float p0 = sc[r], p1 = sc[a.chunk + r];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            o0[j] = fmaf(p0, v8[j], o0[j]);
            o1[j] = fmaf(p1, v8[j], o1[j]);
        }
    }
    store8(red + ((size_t)rg * 2 + 0) * kD + g16 * 8, o0);
    store8(red + ((size_t)rg * 2 + 1) * kD + g16 * 8, o1);
    __syncthreads();

    // Thread t reduces dims (h = t / 64, d = 2*(t % 64) .. +1) over the 8 row groups.
    const int h = tid >> 6;
    const int d = 2 * (tid & 63);
    float ox = 0.f, oy = 0.f;
#pragma unroll
    for (int g = 0; g < 8; g++) {
        const float2 v = *reinterpret_cast<const float2*>(red + ((size_t)g * 2 + h) * kD + d);
        ox += v.x;
        oy += v.y;
    }
    const size_t out_off = (size_t)b * kHq * kD + (size_t)(kGroup * kvh + h) * kD + d;

    if (nsplit == 1) {
        const float inv = 1.f / stat[2 + h];
        *reinterpret_cast<float2*>(a.out + out_off) = make_float2(ox * inv, oy * inv);
        return;
    }

    float* part_base = a.partials + ((size_t)(b * kHkv + kvh) * a.nsplit_max) * 2 * kPartStride;
    {
        float* mine = part_base + ((size_t)s * 2 + h) * kPartStride;
        if ((tid & 63) == 0) {
            mine[0] = stat[h];
            mine[1] = stat[2 + h];
        }
        *reinterpret_cast<float2*>(mine + 4 + d) = make_float2(ox, oy);
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned int ticket = atomicAdd(&a.counters[b * kHkv + kvh], 1u);
        *last_flag = (ticket == (unsigned int)(nsplit - 1));
    }
    __syncthreads();
    if (!*last_flag) return;
    __threadfence();

    // Last CTA of this (sequence, KV head): merge the splits.
    float M = -INFINITY;
    for (int j = 0; j < nsplit; j++) M = fmaxf(M, __ldcg(part_base + ((size_t)j * 2 + h) * kPartStride));
    float L = 0.f, ax = 0.f, ay = 0.f;
    for (int j = 0; j < nsplit; j++) {
        const float* pj = part_base + ((size_t)j * 2 + h) * kPartStride;
        const float w = fast_exp2(__ldcg(pj) - M);
        L = fmaf(__ldcg(pj + 1), w, L);
        const float2 o = __ldcg(reinterpret_cast<const float2*>(pj + 4 + d));
        ax = fmaf(o.x, w, ax);
        ay = fmaf(o.y, w, ay);
    }
    const float inv = 1.f / L;
    *reinterpret_cast<float2*>(a.out + out_off) = make_float2(ax * inv, ay * inv);
    if (tid == 0) a.counters[b * kHkv + kvh] = 0u;
}

template <typename T>
static size_t decode_smem_bytes(int chunk)
{
    return (size_t)2 * chunk * kD * sizeof(T) + sizeof(float) * (2 * chunk + 8 * 2 * kD + 8) +
           2 * sizeof(uint64_t) + 16;
}

template <typename T>
static int launch_decode(const DecodeArgs& a, int batch, void* stream)
{
    const size_t smem = decode_smem_bytes<T>(a.chunk);
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(decode_split_kernel<T>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)decode_smem_bytes<T>(DecodeTile<T>::kMaxChunk));
        if (e != cudaSuccess) return (int)e;
        attr_set = true;
    }
    dim3 grid(a.nsplit_max, kHkv, batch);
    decode_split_kernel<T><<<grid, kDecThreads, smem, (cudaStream_t)stream>>>(a);
    return (int)cudaGetLastError();
}

}  // namespace tyb

using namespace tyb;

extern "C" void tyb_decode_plan(int batch, int max_kv_len, int kv_dtype, int* chunk_rows,
                                int* nsplit)
{
    const int max_chunk =
        kv_dtype == TYB_BF16 ? DecodeTile<__nv_bfloat16>::kMaxChunk : DecodeTile<float>::kMaxChunk;
    // Aim for about four CTAs per SM across the grid (148 SMs), with at least 16 rows per
    // split so each split's copies stay worth their setup.
    const long long target_ctas = 4LL * 148;
    long long per_seq_head = (target_ctas + (long long)batch * kHkv - 1) / ((long long)batch * kHkv);
    if (per_seq_head < 1) per_seq_head = 1;
    long long chunk = (max_kv_len + per_seq_head - 1) / per_seq_head;
    chunk = (chunk + 15) / 16 * 16;
    if (chunk < 16) chunk = 16;
    if (chunk > max_chunk) chunk = max_chunk;
    *chunk_rows = (int)chunk;
    *nsplit = max_kv_len > 0 ? (int)((max_kv_len + chunk - 1) / chunk) : 0;
}

extern "C" size_t tyb_decode_partial_floats(int batch, int nsplit)
{
    return (size_t)batch * kHkv * (size_t)nsplit * 2 * kPartStride;
}

extern "C" int tyb_decode_launch(const float* q, float* out, const tyb_seq_kv* seqs_dev,
                                 tyb_seq_kv one, int batch, int max_kv_len, int kv_dtype,
                                 float scale, float* partials, unsigned int* counters, void* stream)
{
    if (batch <= 0 || max_kv_len <= 0) return 0;
    DecodeArgs a;
    a.q = q;
    a.out = out;
    a.seqs = seqs_dev;
    a.one = one;
    a.scale_log2 = scale * kLog2e;
    int chunk, nsplit;
    tyb_decode_plan(batch, max_kv_len, kv_dtype, &chunk, &nsplit);
    a.chunk = chunk;
    a.nsplit_max = nsplit;
    a.partials = partials;
    a.counters = counters;
    if (kv_dtype == TYB_BF16) return launch_decode<__nv_bfloat16>(a, batch, stream);
    return launch_decode<float>(a, batch, stream);
}
