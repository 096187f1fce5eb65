// prefill_tc32.cu -- causal GQA flash attention for the drop-in FP32 prefill entry points
// (attention_prefill_gqa, attention_chunked_prefill_gqa) on the 5th-generation tensor cores, at
// the FP32 parity bar.
//
// Reference semantics: kernel/attention.c:252-381 (scratch Q/K/V, keys k <= q with the local
// query index, Sk clamping the key range) and :413-543 (keys from the cache, k <= pos_offset + q);
// rows with no visible key give 0 (:347-361).  Inputs arrive already normalised and rotated, as
// kernel/decoder.c:73-93 leaves them.
//
// FP32 accuracy from BF16 tensor cores: every FP32 operand x is carried as a pair of BF16 values
// hi = bf16(x), lo = bf16(x - hi) (x = hi + lo to about 2^-17 relative), and each product as
// three BF16 MMAs with FP32 accumulation, the lo . lo term (2^-18 relative) dropped:
//     S = Qhi.Khi^T + Qhi.Klo^T + Qlo.Khi^T      O += Phi.Vhi + Phi.Vlo + Plo.Vhi
// K and V rows of a BF16 cache are exact in BF16 (lo = 0), so those products take two MMAs.
//
// Work item = 128 query tokens x one query head (grid: q-tiles x 16 heads, longest items
// first).  Warps 0-3 (one TMEM lane = one query row per thread) load the queries and split them
// into the hi / lo tiles, run the online softmax (base 2) and write P as hi / lo BF16 pairs into
// the P columns of its TMEM row, and write the output; warp 4 issues the MMAs from one thread;
// warp 5 streams K and V tiles (hi and lo, 128 keys x 128 dims) by TMA tensor copies.
// Shared memory: Qhi Qlo Khi Klo Vhi Vlo, 32 KB each (one CTA per SM); TMEM: S | O | P (hi, lo),
// 128 columns each of the 512: S is released as soon as the softmax has loaded it, so the next
// tile's QK runs during the softmax (6.84 -> 5.32 ms per config-3 page against P written over S).
// Per tile the chain is QK -> softmax -> P.V; the next tile's K copy runs during the softmax and
// P.V, the next V copy during the next QK and softmax.  Every mbarrier wait is bounded; a timed-out
// CTA raises the status word, leaves its loops, frees its TMEM and returns.
#include <cuda.h>

#define TYB_WHOLE_PROGRAM
#include "common.cuh"
#include "tcgen05.cuh"

namespace tyb {

constexpr int kT32Rows = 128;            // query tokens per item (= tensor-core M)
constexpr int kT32Keys = 128;            // keys per tile
constexpr int kT32Threads = 192;         // warps 0-3 softmax, warp 4 MMA issue, warp 5 TMA
constexpr int kT32Tile = 128 * 128 * 2;  // one 128 x 128 BF16 operand tile: 32 KB
constexpr size_t kT32SmemBytes = 6 * (size_t)kT32Tile + 128 + 1024;  // tiles + barriers + alignment

struct PrefillTc32Args {
    const float* q;        // [Sq][16][128] fp32
    float* out;            // [Sq][16][128] fp32
    int Sq;
    int pos_offset;        // key k is visible to query i iff k <= pos_offset + i ...
    int total_kv;          // ... and k < total_kv (>= 1)
    int n_qtiles;
    int split_kv;          // 1: K and V arrive as hi + lo BF16 tiles; 0: BF16 rows (lo = 0)
    float scale_log2;
    unsigned int* status;  // the library's status word
    unsigned int* mirror;  // its page-locked host mirror flag, or NULL
    unsigned long long wait_ns;  // limit of every bounded wait (tyb_wait_limit)
};

// Largest visible score of a row: columns [0, lim).
template <bool kMask>
__device__ __forceinline__ float t32_row_max(const float (&s)[kT32Keys], int lim)
{
    float m[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
    for (int c = 0; c < kT32Keys; c++) {
        const float x = (!kMask || c < lim) ? s[c] : -INFINITY;
        m[c & 3] = fmaxf(m[c & 3], x);
    }
    return fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3]));
}

// p = exp2(s * scale_log2 + neg_m) on the visible columns (0 elsewhere); P written into this
// row's TMEM columns as BF16 pairs, hi parts in [p_addr, p_addr + 64), lo parts in
// [p_addr + 64, p_addr + 128) (column c / 2 of each half holds keys c, c + 1).  Returns the FP32
// sum of the row's p; the stores are waited for before returning.
template <bool kMask>
__device__ __forceinline__ float t32_row_exp(const float (&s)[kT32Keys], int lim, float scale_log2, float neg_m,
                                             uint32_t p_addr)
{
    const float2 sc = make_float2(scale_log2, scale_log2), nm = make_float2(neg_m, neg_m);
    float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
#pragma unroll
    for (int part = 0; part < 4; part++) {
        uint32_t ph[16], pl[16];
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
            const int k = part * 32 + c;
            float2 x = __ffma2_rn(make_float2(s[k], s[k + 1]), sc, nm);
            if (kMask) {
                if (k >= lim) x.x = -INFINITY;
                if (k + 1 >= lim) x.y = -INFINITY;
            }
            const float2 e = make_float2(pt_exp2(x.x), pt_exp2(x.y));
            if ((c >> 1) & 1) acc1 = __fadd2_rn(acc1, e);
            else acc0 = __fadd2_rn(acc0, e);
            const __nv_bfloat162 hi = __floats2bfloat162_rn(e.x, e.y);
            const float2 hf = __bfloat1622float2(hi);
            ph[c >> 1] = *reinterpret_cast<const uint32_t*>(&hi);
            pl[c >> 1] = pack_bf16x2(e.x - hf.x, e.y - hf.y);
        }
        tmem_st16u(p_addr + part * 16, ph);
        tmem_st16u(p_addr + 64 + part * 16, pl);
    }
    tmem_wait_st();
    return (acc0.x + acc0.y) + (acc1.x + acc1.y);
}

// The item's 128 query rows of head h as hi and lo BF16 tiles in the 128-byte-swizzled K-major
// layout of the QK MMA.  Warp w loads rows 32 w .. 32 w + 31; lane l holds dims [4 l, 4 l + 4).
// Eight rows' loads go out before any is used; rows past Sq are zero.
__device__ __forceinline__ void t32_load_queries(const PrefillTc32Args& a, unsigned char* sQh, unsigned char* sQl,
                                                 int t0, int h, int warp, int lane)
{
#pragma unroll 1
    for (int i0 = 0; i0 < 32; i0 += 8) {
        float4 x[8];
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int tok = t0 + 32 * warp + i0 + u;
            x[u] = tok < a.Sq ? __ldg(reinterpret_cast<const float4*>(a.q + ((size_t)tok * kHq + h) * kD + 4 * lane))
                              : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int r = 32 * warp + i0 + u;
            const __nv_bfloat162 h0 = __floats2bfloat162_rn(x[u].x, x[u].y);
            const __nv_bfloat162 h1 = __floats2bfloat162_rn(x[u].z, x[u].w);
            const float2 f0 = __bfloat1622float2(h0), f1 = __bfloat1622float2(h1);
            const uint2 hi = make_uint2(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1));
            const uint2 lo = make_uint2(pack_bf16x2(x[u].x - f0.x, x[u].y - f0.y), pack_bf16x2(x[u].z - f1.x, x[u].w - f1.y));
            const uint32_t off = sw128_offset(r, 4 * lane);
            *reinterpret_cast<uint2*>(sQh + off) = hi;
            *reinterpret_cast<uint2*>(sQl + off) = lo;
        }
    }
}

__global__ void __launch_bounds__(kT32Threads, 1)
    prefill_tc32_kernel(const __grid_constant__ CUtensorMap tkh, const __grid_constant__ CUtensorMap tkl,
                        const __grid_constant__ CUtensorMap tvh, const __grid_constant__ CUtensorMap tvl,
                        const PrefillTc32Args a)
{
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* sQh = smem;
    unsigned char* sQl = smem + kT32Tile;
    unsigned char* sKh = smem + 2 * kT32Tile;
    unsigned char* sKl = smem + 3 * kT32Tile;
    unsigned char* sVh = smem + 4 * kT32Tile;
    unsigned char* sVl = smem + 5 * kT32Tile;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 6 * kT32Tile);
    uint64_t* q_full = bars + 0;   // query tiles written (128 arrivals)
    uint64_t* k_full = bars + 1;   // K tile landed
    uint64_t* k_free = bars + 2;   // the QK MMAs of the tile have read it
    uint64_t* v_full = bars + 3;   // V tile landed
    uint64_t* v_free = bars + 4;   // the P.V MMAs of the tile have read it
    uint64_t* s_full = bars + 5;   // S of the tile in TMEM (and every earlier MMA complete)
    uint64_t* p_full = bars + 6;   // P written, O rescaled (128 arrivals)
    uint64_t* pv_done = bars + 7;  // P.V of the tile complete
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);
    uint64_t* s_free = bars + 9;   // S of the tile loaded by the softmax (128 arrivals)

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int qt = a.n_qtiles - 1 - (int)blockIdx.x / kHq;  // longest items first
    const int h = (int)blockIdx.x % kHq;
    const int kvh = h / kGroup;
    const int t0 = qt * kT32Rows;
    const int ntok = min(kT32Rows, a.Sq - t0);
    const int last_key = min(a.pos_offset + t0 + ntok - 1, a.total_kv - 1);
    const int ntiles = last_key / kT32Keys + 1;

    if (warp == 4) {
        if (lane == 0) {
            mbar_init(q_full, 128);
            mbar_init(k_full, 1);
            mbar_init(k_free, 1);
            mbar_init(v_full, 1);
            mbar_init(v_free, 1);
            mbar_init(s_full, 1);
            mbar_init(p_full, 128);
            mbar_init(pv_done, 1);
            mbar_init(s_free, 128);
            fence_barrier_init();
            fence_proxy_async_smem();
        }
        __syncwarp();
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        tc_fence_before();
    }
    __syncthreads();  // barriers initialised, TMEM allocated
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // Everything below reads what earlier work in the stream wrote (queries, K/V rows): the CTA
    // may have started early (programmatic dependent launch after the K/V split pass).
    asm volatile("griddepcontrol.wait;" ::: "memory");

    auto wait = [&](uint64_t* bar, uint32_t parity) {
        return mbar_wait_bounded_to(bar, parity, a.wait_ns, TYB_STATUS_WAIT_TIMEOUT, a.status, a.mirror);
    };

    if (warp == 5) {
        // ---- TMA producers: lane 0 streams K, lane 1 V, each single-buffered and refilled once
        // the MMAs of the previous tile have read it (separate lanes: the next K is wanted
        // while the previous V is still being read).
        if (lane < 2) {
            const bool is_v = lane == 1;
            const uint32_t bytes = a.split_kv ? 2u * kT32Tile : (uint32_t)kT32Tile;
            uint64_t* full = is_v ? v_full : k_full;
            uint64_t* free_ = is_v ? v_free : k_free;
            unsigned char* dh = is_v ? sVh : sKh;
            unsigned char* dl = is_v ? sVl : sKl;
            const CUtensorMap* mh = is_v ? &tvh : &tkh;
            const CUtensorMap* ml = is_v ? &tvl : &tkl;
            for (int j = 0; j < ntiles; j++) {
                const int k0 = j * kT32Keys;
                if (j > 0 && !wait(free_, (uint32_t)(j - 1) & 1u)) break;
                mbar_arrive_expect_tx(full, bytes);
                tma_load_3d(dh, mh, 0, k0, kvh, full);
                tma_load_3d(dh + kTcBox, mh, 64, k0, kvh, full);
                if (a.split_kv) {
                    tma_load_3d(dl, ml, 0, k0, kvh, full);
                    tma_load_3d(dl + kTcBox, ml, 64, k0, kvh, full);
                }
            }
        }
        __syncwarp();
    } else if (warp == 4) {
        // ---- MMA issue (one thread) ----
        if (lane == 0) {
            const uint32_t idesc_qk = umma_idesc(false), idesc_pv = umma_idesc(true);
            const uint64_t dqh = umma_desc(smem_u32(sQh), 16), dql = umma_desc(smem_u32(sQl), 16);
            const uint64_t dkh = umma_desc(smem_u32(sKh), 16), dkl = umma_desc(smem_u32(sKl), 16);
            const uint64_t dvh = umma_desc(smem_u32(sVh), kTcBox), dvl = umma_desc(smem_u32(sVl), kTcBox);
            const bool split = a.split_kv != 0;
            // S in TMEM columns 0-127, O in 128-255, P (hi | lo) in 256-383: S is free once the
            // softmax has loaded it, so QK(j + 1) runs during the softmax of tile j and P.V(j)
            // follows once P(j) is written (the softmax writes P(j + 1) after P.V(j)).
            auto qk = [&]() {  // S = Qhi.Khi^T + Qhi.Klo^T + Qlo.Khi^T
#pragma unroll
                for (int kk = 0; kk < 8; kk++) {
                    const uint32_t off = ((kk >> 2) * kTcBox + (kk & 3) * 32) >> 4;
                    tc_mma(tmem, dqh + off, dkh + off, idesc_qk, kk > 0);
                    if (split) tc_mma(tmem, dqh + off, dkl + off, idesc_qk, 1);
                    tc_mma(tmem, dql + off, dkh + off, idesc_qk, 1);
                }
                tc_commit(s_full);
                tc_commit(k_free);
            };
            bool ok = wait(q_full, 0) && wait(k_full, 0);
            if (ok) {
                tc_fence_after();
                qk();
            }
            for (int j = 0; j < ntiles && ok; j++) {
                const uint32_t par = (uint32_t)j & 1u;
                if (j + 1 < ntiles) {
                    ok = wait(s_free, par) && wait(k_full, (uint32_t)(j + 1) & 1u);
                    if (!ok) break;
                    tc_fence_after();
                    qk();
                }
                ok = wait(p_full, par) && wait(v_full, par);
                if (!ok) break;
                tc_fence_after();
                // O += Phi.Vhi + Phi.Vlo + Plo.Vhi, P from TMEM (hi in columns [256, 320), lo in [320, 384))
#pragma unroll
                for (int kk = 0; kk < 8; kk++) {
                    const uint32_t voff = (kk * 16 * 128) >> 4;
                    tc_mma_ts(tmem + 128, tmem + 256 + kk * 8, dvh + voff, idesc_pv, (j > 0 || kk > 0));
                    if (split) tc_mma_ts(tmem + 128, tmem + 256 + kk * 8, dvl + voff, idesc_pv, 1);
                    tc_mma_ts(tmem + 128, tmem + 320 + kk * 8, dvh + voff, idesc_pv, 1);
                }
                tc_commit(v_free);
                tc_commit(pv_done);
            }
        }
        __syncwarp();
    } else {
        // ---- queries, softmax, epilogue: warps 0-3, one row per thread ----
        t32_load_queries(a, sQh, sQl, t0, h, warp, lane);
        fence_proxy_async_smem();  // the tensor core reads Q through the async proxy
        mbar_arrive(q_full);

        const int r = 32 * warp + lane;  // row = TMEM lane = token t0 + r
        const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
        const uint32_t s_addr = tmem + lane_base;
        const uint32_t o_addr = tmem + lane_base + 128;
        const uint32_t p_addr = tmem + lane_base + 256;
        const int qpos = a.pos_offset + t0 + r;
        const int qmin = a.pos_offset + t0;
        float m_run = -INFINITY, l_run = 0.f;
        bool ok = true;
        auto warp_wait = [&](uint64_t* bar, uint32_t parity) {  // warp-uniform (TMEM accesses are collective)
            return !__any_sync(0xffffffffu, !wait(bar, parity));
        };
        for (int j = 0; j < ntiles; j++) {
            if (!warp_wait(s_full, (uint32_t)j & 1u)) {
                ok = false;
                break;
            }
            tc_fence_after();
            float sv[kT32Keys];
            tmem_ld128(s_addr, sv);
            tc_fence_before();
            mbar_arrive(s_free);  // S may take the next tile's QK
            // P is the previous P.V's operand, and O its accumulator, until that P.V completes.
            if (j > 0) {
                if (!warp_wait(pv_done, (uint32_t)(j - 1) & 1u)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
            }
            const int k0 = j * kT32Keys;
            const bool masked = k0 + kT32Keys - 1 > qmin || k0 + kT32Keys > a.total_kv;
            const int lim = masked ? min(qpos, a.total_kv - 1) - k0 + 1 : kT32Keys;  // columns [0, lim) visible
            const float m_tile = (masked ? t32_row_max<true>(sv, lim) : t32_row_max<false>(sv, lim)) * a.scale_log2;
            if (j == 0) {
                m_run = m_tile;
                const float neg_m = m_run == -INFINITY ? 0.f : -m_run;
                l_run = masked ? t32_row_exp<true>(sv, lim, a.scale_log2, neg_m, p_addr)
                               : t32_row_exp<false>(sv, lim, a.scale_log2, neg_m, p_addr);
            } else {
                // The running maximum moves only when the tile's exceeds it by more than 2^8 (P <= 256
                // stays exact in the hi / lo pair), which spares the O rescale on most tiles.
                const bool move = m_tile > m_run + 8.f;
                const float m_new = move ? m_tile : m_run;
                const float alpha = move ? pt_exp2(m_run - m_new) : 1.f;
                const float rowsum = masked ? t32_row_exp<true>(sv, lim, a.scale_log2, -m_new, p_addr)
                                            : t32_row_exp<false>(sv, lim, a.scale_log2, -m_new, p_addr);
                if (__any_sync(0xffffffffu, move)) {  // O is complete up to tile j - 1 (pv_done above)
#pragma unroll
                    for (int q4 = 0; q4 < 4; q4++) {
                        float ov[32];
                        tmem_ld32(o_addr + q4 * 32, ov);
#pragma unroll
                        for (int c = 0; c < 32; c++) ov[c] *= alpha;
                        tmem_st32(o_addr + q4 * 32, ov);
                    }
                    tmem_wait_st();
                }
                l_run = l_run * alpha + rowsum;
                m_run = m_new;
            }
            tc_fence_before();
            mbar_arrive(p_full);
        }
        // Epilogue: O / l for this row (0 for a row that sees no key).
        if (ok && warp_wait(pv_done, (uint32_t)(ntiles - 1) & 1u)) {
            tc_fence_after();
            const int tok = t0 + r;
            const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
            float* dst = a.out + ((size_t)tok * kHq + h) * kD;
#pragma unroll
            for (int c = 0; c < 4; c++) {
                float v[32];
                tmem_ld32(o_addr + c * 32, v);
                if (tok < a.Sq) {
#pragma unroll
                    for (int i = 0; i < 32; i += 4)
                        *reinterpret_cast<float4*>(dst + c * 32 + i) =
                            make_float4(v[i] * inv, v[i + 1] * inv, v[i + 2] * inv, v[i + 3] * inv);
                }
            }
        }
        tc_fence_before();
    }
    __syncthreads();
    if (warp == 4) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
    }
}

// ---- K/V split pass ---------------------------------------------------------------------------
// Rows [0, n) of the 8 KV heads of K and V, FP32 with element (head h, row r, dim d) at
// base + r * row_stride + h * head_stride + d, written as hi = bf16(x) and lo = bf16(x - hi) into
// rows row0 + r of head-first [8][cap][128] BF16 arrays.  One thread per 4 dims of a row of K and
// of V.
__global__ void kv_split_kernel(const float* __restrict__ k, const float* __restrict__ v, long long row_stride,
                                long long head_stride, int n, int row0, int cap, __nv_bfloat16* __restrict__ kh,
                                __nv_bfloat16* __restrict__ kl, __nv_bfloat16* __restrict__ vh,
                                __nv_bfloat16* __restrict__ vl)
{
    // The attention kernel that follows may launch now; it waits for this grid before reading.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const long long total = (long long)n * kHkv * 32;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int q4 = (int)(i & 31);
        const long long rh = i >> 5;  // token-major order: row r, then head hh
        const int hh = (int)(rh % kHkv);
        const int r = (int)(rh / kHkv);
        const size_t src = (size_t)r * row_stride + (size_t)hh * head_stride + 4 * q4;
        const size_t dst = ((size_t)hh * cap + row0 + r) * kD + 4 * q4;
        const float4 xk = __ldg(reinterpret_cast<const float4*>(k + src));
        const float4 xv = __ldg(reinterpret_cast<const float4*>(v + src));
        auto split4 = [](const float4 x, __nv_bfloat16* hi, __nv_bfloat16* lo, size_t off) {
            const __nv_bfloat162 h0 = __floats2bfloat162_rn(x.x, x.y), h1 = __floats2bfloat162_rn(x.z, x.w);
            const float2 f0 = __bfloat1622float2(h0), f1 = __bfloat1622float2(h1);
            *reinterpret_cast<uint2*>(hi + off) =
                make_uint2(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1));
            *reinterpret_cast<uint2*>(lo + off) =
                make_uint2(pack_bf16x2(x.x - f0.x, x.y - f0.y), pack_bf16x2(x.z - f1.x, x.w - f1.y));
        };
        split4(xk, kh, kl, dst);
        split4(xv, vh, vl, dst);
    }
}

}  // namespace tyb

using namespace tyb;

extern "C" int tyb_kv_split_rows_launch(const float* k, const float* v, long long row_stride, long long head_stride,
                                        int n, int row0, int cap, void* kh, void* kl, void* vh, void* vl, void* stream)
{
    if (n <= 0) return 0;
    if (row0 < 0 || row0 + n > cap) return (int)cudaErrorInvalidValue;
    const int threads = 256;
    long long blocks = ((long long)n * kHkv * 32 + threads - 1) / threads;
    if (blocks > 148LL * 8) blocks = 148LL * 8;
    kv_split_kernel<<<(unsigned)blocks, threads, 0, (cudaStream_t)stream>>>(
        k, v, row_stride, head_stride, n, row0, cap, static_cast<__nv_bfloat16*>(kh), static_cast<__nv_bfloat16*>(kl),
        static_cast<__nv_bfloat16*>(vh), static_cast<__nv_bfloat16*>(vl));
    return (int)cudaGetLastError();
}

extern "C" int tyb_kv_split_launch(const float* k, const float* v, long long row_stride, long long head_stride, int n,
                                   void* kh, void* kl, void* vh, void* vl, void* stream)
{
    return tyb_kv_split_rows_launch(k, v, row_stride, head_stride, n, 0, n, kh, kl, vh, vl, stream);
}

extern "C" int tyb_prefill_tc32_launch(const float* q, float* out, int Sq, int pos_offset, int total_kv,
                                       const void* k_hi, const void* k_lo, const void* v_hi, const void* v_lo,
                                       int head_rows, float scale, void* stream)
{
    if (Sq <= 0) return 0;
    if (total_kv <= 0 || !k_hi || !v_hi || (!k_lo) != (!v_lo)) return (int)cudaErrorInvalidValue;
    static bool ready[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= 64) return (int)cudaErrorInvalidDevice;
    if (!ready[dev]) {
        e = cudaFuncSetAttribute(prefill_tc32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kT32SmemBytes);
        if (e != cudaSuccess) return (int)e;
        ready[dev] = true;
    }
    PrefillTc32Args a;
    a.q = q;
    a.out = out;
    a.Sq = Sq;
    a.pos_offset = pos_offset;
    a.total_kv = total_kv;
    a.n_qtiles = (Sq + kT32Rows - 1) / kT32Rows;
    a.split_kv = k_lo ? 1 : 0;
    a.scale_log2 = scale * kLog2e;
    a.status = tyb_status_word();
    if (!a.status) return (int)cudaErrorInvalidSymbol;
    a.mirror = tyb_status_mirror_device();
    a.wait_ns = tyb_wait_limit();
    // K/V: [8 heads][head_rows][128] BF16, rows [0, total_kv) visible to the copies (past it: zeros).
    CUtensorMap mkh, mkl, mvh, mvl;
    if (tyb_encode_rows_map(&mkh, k_hi, total_kv, head_rows, kT32Keys) ||
        tyb_encode_rows_map(&mvh, v_hi, total_kv, head_rows, kT32Keys))
        return (int)cudaErrorInvalidValue;
    if (k_lo) {
        if (tyb_encode_rows_map(&mkl, k_lo, total_kv, head_rows, kT32Keys) ||
            tyb_encode_rows_map(&mvl, v_lo, total_kv, head_rows, kT32Keys))
            return (int)cudaErrorInvalidValue;
    } else {
        mkl = mkh;  // unused
        mvl = mvh;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(a.n_qtiles * kHq));
    cfg.blockDim = dim3(kT32Threads);
    cfg.dynamicSmemBytes = kT32SmemBytes;
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return (int)cudaLaunchKernelEx(&cfg, prefill_tc32_kernel, mkh, mkl, mvh, mvl, a);
}
