// prefill_tc.cu -- causal GQA flash attention for prefill on the 5th-generation tensor
// cores (tcgen05 + TMEM), BF16 operands, FP32 accumulation, with QK-RMSNorm and M-RoPE
// fused into the query load, plus the KV-cache append kernel that normalises and rotates K.
//
// Reference semantics: kernel/decoder.c:73-117 for one layer -- per-head RMSNorm of q and k
// with q_norm/k_norm (kernel/ops.c:22-62), rotate_half M-RoPE with per-token cos/sin
// (kernel/ops.c:297-343), K/V appended to the cache at rows seq_len.. (kernel/kv_cache.c:
// 80-104), then causal attention of the new queries over cache rows [0, seq_len + S) with
// query i at position seq_len + i (kernel/attention.c:413-543; seq_len = 0 is the plain
// prefill of :252-381).
//
// Work item = 128 query tokens x the 2 query heads of one KV head (the GQA pair folded into
// the tile: one K/V tile feeds both heads).  Per item:
//   * all 8 softmax warps load the raw queries, RMSNorm + rotate them in registers and store
//     them as BF16 into shared memory in the 128-byte-swizzled K-major layout the tensor core
//     reads (Q0, Q1: 128 x 128 each);
//   * one thread of warp 9 streams K and V tiles (128 keys x 128 dims, BF16) from the cache
//     with TMA tensor copies (SWIZZLE_128B; rows past the attended length are zero-filled), and
//     one thread of warp 8 issues the MMAs: S = Q_h . K^T into TMEM (the heads in turn), later
//     O_h += P_h . V into TMEM;
//   * softmax warp w owns TMEM lane (row) 32*(w%4)+lane of head w/4: it reads its S row with
//     tcgen05.ld (which frees S for the other head's next QK), applies the causal mask and the
//     online softmax (base 2), rescales its O row in TMEM when the running maximum moves, and
//     writes P as BF16 pairs into its head's P columns of TMEM, where the P.V MMA reads it;
//   * the epilogue reads O, divides by the row sum and writes the output rows (or, sharded,
//     the output tiles to every rank).
// TMEM: S (128 columns, the two heads in turn) | P0 | P1 (64 each) | O0 | O1 (128 each): all 512.
// With one S buffer that each head's softmax releases as soon as it has read it, a head's next QK
// needs no wait for its P.V (P has columns of its own), so the QK -> softmax -> P.V chain of a
// head no longer sets the period: 2.39 -> 2.31 ms per config-3 page against an S per head with P
// written over it.  Shared memory: Q0 Q1, K stages 0-1,
// V stages 0-1, 32 KB each.  Every mbarrier wait is bounded; a timed-out CTA raises the status word, leaves its
// loops, frees its TMEM and returns.
#include <cuda.h>

#define TYB_WHOLE_PROGRAM
#include "common.cuh"
#include "tcgen05.cuh"

namespace tyb {

constexpr int kPtRows = 128;            // query tokens per item (= tensor-core M)
constexpr int kPtKeys = 128;            // keys per tile (= N of S, K of P.V)
constexpr int kPtSoftmaxThreads = 256;  // warpgroups 0, 1 (warps 0-3 head 0, 4-7 head 1)
constexpr int kPtThreads = kPtSoftmaxThreads + 128;  // + warpgroup 2: warp 8 MMA issue, warp 9 TMA
// Register split (setmaxnreg): the kernel is launched at kPtLaunchRegs per thread; the issue
// warpgroup drops to kPtIssueRegs and the two softmax warpgroups rise to kPtSoftmaxRegs, so
// that a softmax thread keeps its 128-column S row in registers with room to spare.  The
// shares fit the launch's registers (checked against the compiled count before launching),
// and a warp of each warpgroup shares every sub-partition's 512 registers per lane.
constexpr int kPtLaunchRegs = 168;
constexpr int kPtIssueRegs = 112;
constexpr int kPtSoftmaxRegs = 192;
static_assert(kPtSoftmaxThreads * kPtSoftmaxRegs + 128 * kPtIssueRegs <= kPtThreads * kPtLaunchRegs,
              "register split exceeds the launch allocation");
static_assert(2 * kPtSoftmaxRegs + kPtIssueRegs <= 512, "register split exceeds a sub-partition");
constexpr int kPtTile = 128 * 128 * 2;  // one 128x128 BF16 operand tile: 32 KB
constexpr int kPtBox = kTcBox;          // one 128-row x 64-column swizzled box: 16 KB

struct PrefillTcArgs {
    const void* q;        // [Sq][16][128] raw queries, fp32 (q_bf16 = 0) or bf16
    int q_bf16;
    const float* q_norm;  // [128]
    const float* cos;     // [Sq][64]
    const float* sin;     // [Sq][64]
    void* out;            // [Sq][16][128], fp32 (out_bf16 = 0) or bf16
    int out_bf16;
    int Sq;
    int pos_offset;       // absolute position of query 0 (rows already in the cache)
    int total_kv;         // pos_offset + Sq: rows attended by the last query
    int n_qtiles;
    float scale_log2;
    float eps;
    int kvh0;              // KV heads [kvh0, kvh0 + nkvh) (and their query heads) are computed
    int nkvh;
    int out_head_major;    // output [2 nkvh][Sq][128] (a contiguous head shard) instead of [Sq][16][128]
    const tyb_prefill_x* xchg;  // non-NULL: BF16 rows into every rank's exchange slot (KV-head sharding)
    unsigned int epoch;    // the call's number (1, 2, ...): slot epoch & 1, flags compared to it
    unsigned int* status;  // the library's status word (tyb_status_word)
    unsigned int* mirror;  // its page-locked host mirror flag (tyb_status_mirror_device), or NULL
    unsigned long long wait_ns;  // limit of every bounded wait (tyb_wait_limit)
};

// Sharded form: per rank, a 4-D map of its exchange slots {128 dims, 16 heads, max_tokens tokens,
// 2 slots} (BF16, token-major), stored to in boxes of {64 dims, 1 head, 128 tokens, 1 slot} with
// the 128-byte swizzle -- the layout of a query tile in shared memory.  Built once per set-up
// (tyb_prefill_x_maps); unused otherwise.
struct PrefillPeerMaps {
    CUtensorMap m[8];
};

// Softmax weight split between the two exp2 units: of every four column pairs of an unmasked
// tile, kPtEmuPairs are evaluated on the FMA pipe (exp2_fma2) and the rest on the MUFU.
constexpr int kPtEmuPairs = 0;
// BF16 packing of P by integer round-half-up (IADD + PRMT) instead of the conversion unit.
constexpr bool kPtIntPack = false;

// Two BF16 values (round to nearest, ties away from zero) from non-negative finite floats.
__device__ __forceinline__ uint32_t pack_bf16x2_rna(float lo, float hi)
{
    return __byte_perm(__float_as_uint(lo) + 0x8000u, __float_as_uint(hi) + 0x8000u, 0x7632);
}

// 2^x of two values on the FMA pipe, for x <= 8 (x below -120 is taken as -120: 2^-120 is
// far below any row sum here).  x = j + f, j = round(x) by the 1.5 * 2^23 shifter, f in
// [-1/2, 1/2]; 2^f by a cubic fitted to minimise the relative error on that interval
// (Lawson's iteratively reweighted least squares, max relative error 7.5e-5 after FP32
// rounding, well inside BF16's 2^-9); 2^j enters through the exponent field.
__device__ __forceinline__ float2 exp2_fma2(float2 x)
{
    x.x = fmaxf(x.x, -120.f);
    x.y = fmaxf(x.y, -120.f);
    const float2 t = __fadd2_rn(x, make_float2(12582912.f, 12582912.f));
    const float2 j = __fadd2_rn(t, make_float2(-12582912.f, -12582912.f));
    const float2 f = __ffma2_rn(j, make_float2(-1.f, -1.f), x);
    float2 p = __ffma2_rn(make_float2(0.055171434f, 0.055171434f), f, make_float2(0.24261081f, 0.24261081f));
    p = __ffma2_rn(p, f, make_float2(0.69326097f, 0.69326097f));
    p = __ffma2_rn(p, f, make_float2(0.99992812f, 0.99992812f));
    return make_float2(__int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23)),
                       __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23)));
}

__device__ __forceinline__ float fmax3(float a, float b, float c)
{
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// Largest visible score of a row: columns [0, lim) (all 128 when the tile needs no mask).
template <bool kMask>
__device__ __forceinline__ float row_max(const float (&s)[kPtKeys], int lim)
{
    float m[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
    for (int c = 0; c < kPtKeys; c += 2) {
        const float a = (!kMask || c < lim) ? s[c] : -INFINITY;
        const float b = (!kMask || c + 1 < lim) ? s[c + 1] : -INFINITY;
        m[(c >> 1) & 3] = fmax3(m[(c >> 1) & 3], a, b);
    }
    return fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3]));
}

// p = exp2(s * scale_log2 + neg_m) on the visible columns (0 on the others), packed as BF16
// pairs into TMEM columns [p_addr, p_addr + 64) of this row (column c / 2 holds keys c, c + 1);
// returns the FP32 sum of the row's p.  The affine step and the sum run two columns per
// instruction (f32x2).  The stores are waited for before returning.
// With kTrack, *xmax receives the largest exponent s * scale_log2 + neg_m of the row.
template <bool kMask, bool kTrack>
__device__ __forceinline__ float row_exp(const float (&s)[kPtKeys], int lim, float scale_log2, float neg_m,
                                         uint32_t p_addr, float* xmax)
{
    const float2 sc = make_float2(scale_log2, scale_log2), nm = make_float2(neg_m, neg_m);
    float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
    float xm0 = -INFINITY, xm1 = -INFINITY;
#pragma unroll
    for (int hf = 0; hf < 4; hf++) {
        uint32_t pk[16];
#pragma unroll
        for (int c = 0; c < 32; c += 4) {
            const int k = hf * 32 + c;
            float2 x0 = __ffma2_rn(make_float2(s[k], s[k + 1]), sc, nm);
            float2 x1 = __ffma2_rn(make_float2(s[k + 2], s[k + 3]), sc, nm);
            if (kMask) {
                if (k >= lim) x0.x = -INFINITY;
                if (k + 1 >= lim) x0.y = -INFINITY;
                if (k + 2 >= lim) x1.x = -INFINITY;
                if (k + 3 >= lim) x1.y = -INFINITY;
            }
            if (kTrack) {
                xm0 = fmax3(xm0, x0.x, x0.y);
                xm1 = fmax3(xm1, x1.x, x1.y);
            }
            const int pair = (c >> 1) & 3;  // pairs c/2, c/2 + 1 of the group of four
            const float2 e0 = (!kMask && pair < kPtEmuPairs) ? exp2_fma2(x0)
                                                            : make_float2(pt_exp2(x0.x), pt_exp2(x0.y));
            const float2 e1 = (!kMask && pair + 1 < kPtEmuPairs) ? exp2_fma2(x1)
                                                                : make_float2(pt_exp2(x1.x), pt_exp2(x1.y));
            acc0 = __fadd2_rn(acc0, e0);
            acc1 = __fadd2_rn(acc1, e1);
            pk[c / 2] = kPtIntPack ? pack_bf16x2_rna(e0.x, e0.y) : pack_bf16x2(e0.x, e0.y);
            pk[c / 2 + 1] = kPtIntPack ? pack_bf16x2_rna(e1.x, e1.y) : pack_bf16x2(e1.x, e1.y);
        }
        tmem_st16u(p_addr + hf * 16, pk);
    }
    tmem_wait_st();
    if (kTrack) *xmax = fmaxf(xm0, xm1);
    return (acc0.x + acc0.y) + (acc1.x + acc1.y);
}

// Query rows of one item into shared memory: RMSNorm(q_norm) + rotate_half M-RoPE, rounded to
// BF16, in the 128-byte-swizzled K-major layout of the QK MMA.  Warp w handles tokens 16w .. +16
// of the item, both query heads of each (they share the token's cos/sin), eight tokens at a
// time; lane l holds dims [4l, 4l + 4) mod 64 of the lower (l < 16) or upper half.  All loads of
// the eight tokens go out before any is used (tokens past Sq read token Sq - 1 and are zeroed),
// so that their latencies overlap: two round trips to memory per warp.
template <bool kBf16>
__device__ __forceinline__ void load_queries(const PrefillTcArgs& a, unsigned char* sQ, int t0, int kvh, int warp,
                                             int lane)
{
    const float4 w = *reinterpret_cast<const float4*>(a.q_norm + 4 * lane);
    const int jr = 4 * (lane & 15);  // rotary frequency index of this lane's first dim
#pragma unroll 1
    for (int i0 = 0; i0 < 16; i0 += 8) {
        float x[8][kGroup][4];
        float4 cv[8], sn[8];
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int tok = min(t0 + 16 * warp + i0 + u, a.Sq - 1);
#pragma unroll
            for (int hh = 0; hh < kGroup; hh++) {
                const size_t off = ((size_t)tok * kHq + kGroup * kvh + hh) * kD + 4 * lane;
                if (kBf16) {
                    const uint2 q2 = __ldg(reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(a.q) + off));
                    const float2 f0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&q2.x));
                    const float2 f1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&q2.y));
                    x[u][hh][0] = f0.x; x[u][hh][1] = f0.y; x[u][hh][2] = f1.x; x[u][hh][3] = f1.y;
                } else {
                    const float4 f = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(a.q) + off));
                    x[u][hh][0] = f.x; x[u][hh][1] = f.y; x[u][hh][2] = f.z; x[u][hh][3] = f.w;
                }
            }
            cv[u] = __ldg(reinterpret_cast<const float4*>(a.cos + (size_t)tok * 64 + jr));
            sn[u] = __ldg(reinterpret_cast<const float4*>(a.sin + (size_t)tok * 64 + jr));
        }
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int r = 16 * warp + i0 + u;
            const bool live = t0 + r < a.Sq;
            const float c4[4] = {cv[u].x, cv[u].y, cv[u].z, cv[u].w};
            const float s4[4] = {sn[u].x, sn[u].y, sn[u].z, sn[u].w};
#pragma unroll
            for (int hh = 0; hh < kGroup; hh++) {
                float ss = x[u][hh][0] * x[u][hh][0] + x[u][hh][1] * x[u][hh][1] + x[u][hh][2] * x[u][hh][2] +
                           x[u][hh][3] * x[u][hh][3];
#pragma unroll
                for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
                const float rs = live ? rsqrtf(ss * (1.f / kD) + a.eps) : 0.f;
                const float y[4] = {x[u][hh][0] * rs * w.x, x[u][hh][1] * rs * w.y, x[u][hh][2] * rs * w.z,
                                    x[u][hh][3] * rs * w.w};
                // rotate_half: lane l < 16 holds dims [4l, 4l+4), lane l+16 the partner dims + 64.
                float partner[4];
#pragma unroll
                for (int e = 0; e < 4; e++) partner[e] = __shfl_xor_sync(0xffffffffu, y[e], 16);
                float z[4];
#pragma unroll
                for (int e = 0; e < 4; e++)
                    z[e] = lane < 16 ? y[e] * c4[e] - partner[e] * s4[e]   // x[j] c - x[j+64] s
                                     : y[e] * c4[e] + partner[e] * s4[e];  // x[j+64] c + x[j] s
                const uint2 packed = make_uint2(pack_bf16x2(z[0], z[1]), pack_bf16x2(z[2], z[3]));
                *reinterpret_cast<uint2*>(sQ + hh * kPtTile + sw128_offset(r, 4 * lane)) = packed;
            }
        }
    }
}

// Barrier of the 128 softmax threads of head h (named barriers 1 and 2; 0 is __syncthreads).
__device__ __forceinline__ void head_bar(int h)
{
    if (h == 0)
        asm volatile("bar.sync 1, 128;" ::: "memory");
    else
        asm volatile("bar.sync 2, 128;" ::: "memory");
}

// 384 threads (3 warpgroups) launched at 168 registers, split 192 / 192 / 112 by setmaxnreg.
__global__ void __launch_bounds__(kPtThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                      const PrefillTcArgs a, const __grid_constant__ PrefillPeerMaps px)
{
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // 1024-byte alignment is required by the 128-byte swizzle atoms.
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* sQ = smem;                  // Q0, Q1
    unsigned char* sK = smem + 2 * kPtTile;    // K stages 0, 1
    unsigned char* sV = smem + 4 * kPtTile;    // V stages 0, 1
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 6 * kPtTile);
    uint64_t* v_full = bars + 0;    // [2] V stage landed
    uint64_t* v_free = bars + 2;    // [2] both P.Vs of the tile in that stage have read it
    uint64_t* k_full = bars + 4;    // [2] K stage landed
    uint64_t* k_free = bars + 6;    // [2] both QKs of the tile in that stage have read it
    uint64_t* s_full = bars + 8;    // [2] per head: S of the tile is in TMEM
    uint64_t* p_full = bars + 10;   // [2] per head: P written, O rescaled (128 arrivals)
    uint64_t* pv_done = bars + 12;  // [2] per head: P.V of the tile finished
    uint64_t* q_full = bars + 14;   // Q0, Q1 written (256 arrivals)
    uint64_t* s_free = bars + 15;   // [2] per head: the softmax has loaded S (128 arrivals)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);  // (bars 15-16: s_free)
    int* store_fail = reinterpret_cast<int*>(bars + 18);  // [2] per head: its output tile is incomplete

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // Longest items first: q-tile index descends with blockIdx.
    const int item = blockIdx.x;
    const int qt = a.n_qtiles - 1 - item / a.nkvh;
    const int kvh = a.kvh0 + item % a.nkvh;
    const int t0 = qt * kPtRows;
    const int ntok = min(kPtRows, a.Sq - t0);
    const int last_pos = a.pos_offset + t0 + ntok - 1;
    const int ntiles = last_pos / kPtKeys + 1;

    if (warp == 8) {
        if (lane == 0) {
            for (int i = 0; i < 2; i++) {
                mbar_init(&v_full[i], 1);
                mbar_init(&v_free[i], 1);
                mbar_init(&s_full[i], 1);
                mbar_init(&p_full[i], kPtSoftmaxThreads / 2);
                mbar_init(&pv_done[i], 1);
                mbar_init(&s_free[i], kPtSoftmaxThreads / 2);
                mbar_init(&k_full[i], 1);
                mbar_init(&k_free[i], 1);
            }
            mbar_init(q_full, kPtSoftmaxThreads);
            store_fail[0] = store_fail[1] = 0;
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

    const uint32_t idesc_qk = umma_idesc(false);
    const uint32_t idesc_pv = umma_idesc(true);

    if (warp >= 8) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kPtIssueRegs));
        if (warp == 9) {
            // ---- TMA producer (one thread): K and V double-buffered, each stage refilled as soon
            // as the MMAs of the tile two back have read it.  The kernel may start while the
            // previous kernel in the stream (kv_prep, which writes the rows read here) still runs:
            // this thread, the only reader of those rows, waits for it first.  Past that wait the
            // CTA lets the next kernel in the stream launch (the next layer's kv_prep, or a decode
            // step): it starts once every CTA of this grid has started and passed the wait -- no
            // CTA of this grid is left waiting for an SM, and kv_prep has completed -- and it
            // waits for this grid before reading anything.
            if (lane == 0) {
                asm volatile("griddepcontrol.wait;" ::: "memory");
                asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
                for (int j = 0; j < ntiles; j++) {
                    const int st = j & 1;
                    const uint32_t fpar = (uint32_t)((j - 2) >> 1) & 1u;
                    if (j >= 2 && !mbar_wait_bounded_to(&k_free[st], fpar, a.wait_ns, TYB_STATUS_WAIT_TIMEOUT, a.status, a.mirror)) break;
                    mbar_arrive_expect_tx(&k_full[st], kPtTile);
                    tma_load_3d(sK + st * kPtTile, &tmap_k, 0, j * kPtKeys, kvh, &k_full[st]);
                    tma_load_3d(sK + st * kPtTile + kPtBox, &tmap_k, 64, j * kPtKeys, kvh, &k_full[st]);
                    if (j >= 2 && !mbar_wait_bounded_to(&v_free[st], fpar, a.wait_ns, TYB_STATUS_WAIT_TIMEOUT, a.status, a.mirror)) break;
                    mbar_arrive_expect_tx(&v_full[st], kPtTile);
                    tma_load_3d(sV + st * kPtTile, &tmap_v, 0, j * kPtKeys, kvh, &v_full[st]);
                    tma_load_3d(sV + st * kPtTile + kPtBox, &tmap_v, 64, j * kPtKeys, kvh, &v_full[st]);
                }
            }
            __syncwarp();
        } else if (warp == 8) {
            // ---- MMA issue (one thread); the two heads ping-pong so that one head's softmax
            // overlaps the other head's tensor-core work.
            if (lane == 0) {
                // Descriptors of the shared-memory operand tiles, built once; a K step of 16 columns
                // within a 128-byte swizzle atom (32 bytes) or the next 64-column box adds to the
                // start address field (16-byte units; shared addresses stay below 2^18: no carry).
                const uint64_t dq0 = umma_desc(smem_u32(sQ), 16), dq1 = umma_desc(smem_u32(sQ) + kPtTile, 16);
                const uint64_t dk0 = umma_desc(smem_u32(sK), 16), dk1 = umma_desc(smem_u32(sK) + kPtTile, 16);
                const uint64_t dv0 = umma_desc(smem_u32(sV), kPtBox), dv1 = umma_desc(smem_u32(sV) + kPtTile, kPtBox);
                auto qk = [&](int h, int j) {  // S = Q_h . K(j)^T (the shared S buffer)
                    const uint64_t dq = h ? dq1 : dq0;
                    const uint64_t dk = (j & 1) ? dk1 : dk0;
    #pragma unroll
                    for (int kk = 0; kk < 8; kk++) {
                        const uint32_t off = ((kk >> 2) * kPtBox + (kk & 3) * 32) >> 4;
                        tc_mma(tmem, dq + off, dk + off, idesc_qk, kk > 0);
                    }
                    tc_commit(&s_full[h]);
                };
                auto pv = [&](int h, int j) {  // O_h += P_h . V(j), P_h (BF16) in TMEM columns 128 + 64 h
                    const uint64_t dv = (j & 1) ? dv1 : dv0;
    #pragma unroll
                    for (int kk = 0; kk < 8; kk++)
                        tc_mma_ts(tmem + 256 + h * 128, tmem + 128 + h * 64 + kk * 8, dv + ((kk * 16 * 128) >> 4), idesc_pv,
                                  (j > 0 || kk > 0));
                    tc_commit(&pv_done[h]);
                };
                auto wait = [&](uint64_t* bar, uint32_t parity) {
                    const bool ok = mbar_wait_bounded_to(bar, parity, a.wait_ns, TYB_STATUS_WAIT_TIMEOUT, a.status, a.mirror);
                    tc_fence_after();
                    return ok;
                };
                // One S buffer (TMEM columns 0-127) for both heads, free as soon as the softmax has
                // loaded it; P_h in columns 128 + 64 h.  So QK(h, j + 1) does not wait for P.V(h, j):
                // head 0's next S is computed once head 1 has loaded its S of tile j, and the P.V of
                // a head follows its P.  (The softmax writes P_h(j + 1) once P.V(h, j) is done.)
                bool ok = wait(q_full, 0) && wait(&k_full[0], 0);
                if (ok) {
                    qk(0, 0);
                    ok = wait(&s_free[0], 0);
                }
                if (ok) {
                    qk(1, 0);
                    tc_commit(&k_free[0]);
                }
                for (int j = 0; j < ntiles && ok; j++) {
                    const uint32_t par = (uint32_t)j & 1u;
                    const bool more = j + 1 < ntiles;
                    const int nst = (j + 1) & 1;
                    if (more) {
                        ok = wait(&s_free[1], par) && wait(&k_full[nst], (uint32_t)((j + 1) >> 1) & 1u);
                        if (!ok) break;
                        qk(0, j + 1);
                    }
                    ok = wait(&p_full[0], par) && wait(&v_full[j & 1], (uint32_t)(j >> 1) & 1u);
                    if (!ok) break;
                    pv(0, j);
                    if (more) {
                        ok = wait(&s_free[0], (uint32_t)(j + 1) & 1u);
                        if (!ok) break;
                        qk(1, j + 1);
                        tc_commit(&k_free[nst]);
                    }
                    ok = wait(&p_full[1], par);
                    if (!ok) break;
                    pv(1, j);
                    tc_commit(&v_free[j & 1]);
                }
            }
            __syncwarp();
        }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kPtSoftmaxRegs));
        // ---- queries: RMSNorm(q_norm) + rotate_half M-RoPE, BF16, swizzled into Q0/Q1 ----------
        // Warps 0-7 (warp w: tokens 16w .. +16, both heads), while the producer already streams
        // the first K/V tiles.
        {
            if (a.q_bf16) load_queries<true>(a, sQ, t0, kvh, warp, lane);
            else load_queries<false>(a, sQ, t0, kvh, warp, lane);
            fence_proxy_async_smem();  // Q is read by the tensor core (async proxy)
            mbar_arrive(q_full);
        }

        // ---- softmax + epilogue: one TMEM lane (row) per thread -----------------------------
        const int h = warp >> 2;
        const int r = 32 * (warp & 3) + lane;  // row = TMEM lane = token t0 + r
        const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
        const uint32_t s_addr = tmem + lane_base;                 // S: one buffer, both heads
        const uint32_t p_addr = tmem + lane_base + 128 + h * 64;  // P_h (BF16 pairs)
        const uint32_t o_addr = tmem + lane_base + 256 + h * 128;
        const int qpos = a.pos_offset + t0 + r;
        const int qmin = a.pos_offset + t0;  // first query position of the item
        float m_run = -INFINITY, l_run = 0.f;
        bool ok = true;
        // A wait that runs out of time ends the loop for the whole warp (the TMEM loads below are
        // warp-collective).
        auto warp_wait = [&](uint64_t* bar, uint32_t parity) {
            return !__any_sync(0xffffffffu,
                               !mbar_wait_bounded_to(bar, parity, a.wait_ns, TYB_STATUS_WAIT_TIMEOUT, a.status, a.mirror));
        };
        for (int j = 0; j < ntiles; j++) {
            const uint32_t par = (uint32_t)j & 1u;
            if (!warp_wait(&s_full[h], par)) {
                ok = false;
                break;
            }
            tc_fence_after();
            float sv[kPtKeys];  // this row of S
            tmem_ld128(s_addr, sv);
            tc_fence_before();
            mbar_arrive(&s_free[h]);  // S may take the other head's next tile
            // P_h is the previous P.V's operand until that P.V completes.
            if (j > 0) {
                if (!warp_wait(&pv_done[h], (uint32_t)(j - 1) & 1u)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
            }
            // Causal mask (key k visible to query qpos iff k <= qpos, and k < total_kv) --
            // only tiles that reach past the item's first query or the attended length need it.
            const int k0 = j * kPtKeys;
            const bool masked = k0 + kPtKeys - 1 > qmin || k0 + kPtKeys > a.total_kv;
            const int lim = masked ? min(qpos, a.total_kv - 1) - k0 + 1 : kPtKeys;  // columns [0, lim) visible
            // The two heads' passes run when their S is ready, sharing the exponential unit (a
            // warp of each per sub-partition).  Making them take turns on it (head 0's tile j
            // after head 1's tile j - 1) measured 1.5 % slower per page.
            if (j == 0) {
                // First tile: the row maximum starts the running one (every row sees key 0).
                m_run = (masked ? row_max<true>(sv, lim) : row_max<false>(sv, lim)) * a.scale_log2;
                const float neg_m = m_run == -INFINITY ? 0.f : -m_run;
                l_run = masked ? row_exp<true, false>(sv, lim, a.scale_log2, neg_m, p_addr, nullptr)
                               : row_exp<false, false>(sv, lim, a.scale_log2, neg_m, p_addr, nullptr);
            } else {
                // Later tiles: the running maximum moves only when the tile's exceeds it by more
                // than 2^8; below that the stale one stays (P <= 256: exact in BF16's range and
                // harmless to the FP32 sums), which spares the O rescale on almost every tile.
                // Exponentials against the running maximum, tracking the largest exponent; only if
                // it passes 8 (P above 2^8) for some row of the warp is the tile redone against the
                // row's new maximum (the same P as taking the tile maximum first: 2.50 against
                // 2.55 ms per page, the separate maximum pass gone from almost every tile).
                float xmax;
                float rowsum = masked ? row_exp<true, true>(sv, lim, a.scale_log2, -m_run, p_addr, &xmax)
                                      : row_exp<false, true>(sv, lim, a.scale_log2, -m_run, p_addr, &xmax);
                const bool move = xmax > 8.f;
                float m_new = m_run, alpha = 1.f;
                if (__any_sync(0xffffffffu, move)) {
                    if (move) {
                        m_new = m_run + xmax;
                        alpha = pt_exp2(m_run - m_new);
                    }
                    rowsum = masked ? row_exp<true, false>(sv, lim, a.scale_log2, -m_new, p_addr, nullptr)
                                    : row_exp<false, false>(sv, lim, a.scale_log2, -m_new, p_addr, nullptr);
                }
                // O rescale: the TMEM accesses are warp-collective, so the warp takes the branch
                // if any of its rows moved (the others multiply by 1).
                if (__any_sync(0xffffffffu, move)) {
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
            mbar_arrive(&p_full[h]);
        }
        // Epilogue: O / l for this row.
        if (a.xchg) {
            // Sharded: the row, BF16, into this head's query tile -- free, since the last QK of
            // the head completed before its last P.V -- in the swizzled layout; then one thread
            // per head sends the 128 x 128 tile to every rank's exchange slot with TMA stores
            // (two 64-dimension boxes per rank), the all-gather of the head outputs done by the
            // epilogue that produces them, in transfers of whole tiles.
            const bool done = ok && warp_wait(&pv_done[h], (uint32_t)(ntiles - 1) & 1u);
            if (!done) {
                store_fail[h] = 1;
            } else {
                tc_fence_after();
                const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
                unsigned char* tile = sQ + h * kPtTile;
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    float v[32];
                    tmem_ld32(o_addr + c * 32, v);
#pragma unroll
                    for (int i = 0; i < 32; i += 8)
                        *reinterpret_cast<uint4*>(tile + sw128_offset(r, c * 32 + i)) =
                            make_uint4(pack_bf16x2(v[i] * inv, v[i + 1] * inv), pack_bf16x2(v[i + 2] * inv, v[i + 3] * inv),
                                       pack_bf16x2(v[i + 4] * inv, v[i + 5] * inv), pack_bf16x2(v[i + 6] * inv, v[i + 7] * inv));
                }
            }
            fence_proxy_async_smem();  // the tile is read by the TMA unit (async proxy)
            head_bar(h);
            if (lane == 0 && (warp & 3) == 0 && !store_fail[h]) {
                const int slot = (int)(a.epoch & 1u), world = a.xchg->world;
                const unsigned char* tile = sQ + h * kPtTile;
#pragma unroll 1
                for (int p = 0; p < world; p++) {
                    tma_store_4d(&px.m[p], 0, kGroup * kvh + h, t0, slot, tile);
                    tma_store_4d(&px.m[p], 64, kGroup * kvh + h, t0, slot, tile + kPtBox);
                }
                tma_store_drain();
                asm volatile("fence.acq_rel.sys;" ::: "memory");
            }
        } else if (ok && warp_wait(&pv_done[h], (uint32_t)(ntiles - 1) & 1u)) {
            tc_fence_after();
            const int tok = t0 + r;
            const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
            const size_t ooff = a.out_head_major
                                    ? ((size_t)(kGroup * (kvh - a.kvh0) + h) * a.Sq + tok) * kD
                                    : ((size_t)tok * kHq + kGroup * kvh + h) * kD;
#pragma unroll
            for (int c = 0; c < 4; c++) {
                float v[32];
                tmem_ld32(o_addr + c * 32, v);
                if (tok < a.Sq) {
                    if (a.out_bf16) {
                        __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(a.out) + ooff + c * 32;
#pragma unroll
                        for (int i = 0; i < 32; i += 8) {
                            const uint4 u = make_uint4(pack_bf16x2(v[i] * inv, v[i + 1] * inv),
                                                       pack_bf16x2(v[i + 2] * inv, v[i + 3] * inv),
                                                       pack_bf16x2(v[i + 4] * inv, v[i + 5] * inv),
                                                       pack_bf16x2(v[i + 6] * inv, v[i + 7] * inv));
                            *reinterpret_cast<uint4*>(dst + i) = u;
                        }
                    } else {
                        float* dst = static_cast<float*>(a.out) + ooff + c * 32;
#pragma unroll
                        for (int i = 0; i < 32; i += 4)
                            *reinterpret_cast<float4*>(dst + i) =
                                make_float4(v[i] * inv, v[i + 1] * inv, v[i + 2] * inv, v[i + 3] * inv);
                    }
                }
            }
        }
        tc_fence_before();
    }
    __syncthreads();
    if (warp == 8) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
    }
    if (a.xchg && tid == 0) {
        // Sharded completion: one system-scope release fence makes this CTA's peer stores (its
        // threads' own through the barrier above) visible before its count; the rank's last item
        // raises the rank's flag in every buffer, then waits -- bounded -- for every rank's flag
        // of this call in its own buffer.  The kernel ends once the assembled output is here.
        unsigned int* hdr = static_cast<unsigned int*>(a.xchg->base[a.xchg->rank]);
        asm volatile("fence.acq_rel.sys;" ::: "memory");
        unsigned int t;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(t) : "l"(hdr + 8) : "memory");
        if (t == gridDim.x - 1) {
            hdr[8] = 0u;  // the next call's counts come after this kernel has completed
            asm volatile("fence.acq_rel.sys;" ::: "memory");
            for (int p = 0; p < a.xchg->world; p++) {
                unsigned int* f = static_cast<unsigned int*>(a.xchg->base[p]) + a.xchg->rank;
                asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(f), "r"(a.epoch) : "memory");
            }
            const uint64_t t0 = globaltimer_ns();
            for (int r = 0; r < a.xchg->world; r++) {
                unsigned int seen;
                while (true) {
                    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(seen) : "l"(hdr + r) : "memory");
                    if ((int)(seen - a.epoch) >= 0) break;
                    if (globaltimer_ns() - t0 > a.wait_ns) {
                        atomicOr(a.status, TYB_STATUS_WAIT_TIMEOUT);
                        flag_mirror(a.mirror);
                        r = a.xchg->world;
                        break;
                    }
                    __nanosleep(64);
                }
            }
        }
    }
}

// ---- K/V append with QK-RMSNorm + M-RoPE on K ------------------------------------------------
// One warp per (token, KV head): RMSNorm(k_norm) + rotate_half with the token's cos/sin, K and V
// written as BF16 into cache rows pos0 + t (layout of tyb_seq_kv).  Launched as a programmatic
// dependent of the previous kernel in the stream: every CTA waits for it before reading anything,
// and only then lets the attention kernel that follows launch -- so that when that kernel's CTAs
// start (reading q, q_norm, cos and sin before their own wait), everything before this kernel has
// completed.
__global__ void kv_prep_kernel(const void* __restrict__ k_raw, const void* __restrict__ v_raw, int in_bf16,
                               const float* __restrict__ k_norm, const float* __restrict__ cosv,
                               const float* __restrict__ sinv, __nv_bfloat16* __restrict__ k_dst,
                               __nv_bfloat16* __restrict__ v_dst, int row_capacity, int pos0, int S, float eps,
                               int kvh0, int nkvh)
{
    const int lane = threadIdx.x & 31;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // 32-bit indices (S * nkvh < 2^21): a 64-bit division per row cost more issue slots than the
    // row's arithmetic.
    const int nwarps = (int)gridDim.x * (int)(blockDim.x >> 5);
    const float4 w = *reinterpret_cast<const float4*>(k_norm + 4 * lane);
    const float w4[4] = {w.x, w.y, w.z, w.w};
    const int jr = 4 * (lane & 15);
    for (int wi = (int)blockIdx.x * (int)(blockDim.x >> 5) + (int)(threadIdx.x >> 5); wi < S * nkvh; wi += nwarps) {
        const int t = wi / nkvh, hh = kvh0 + (wi - t * nkvh);
        const size_t off = ((size_t)t * kHkv + hh) * kD + 4 * lane;
        float x[4], v4[4];
        if (in_bf16) {
            const uint2 uk = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(k_raw) + off);
            const uint2 uv = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(v_raw) + off);
            const __nv_bfloat162* hk = reinterpret_cast<const __nv_bfloat162*>(&uk);
            const __nv_bfloat162* hv = reinterpret_cast<const __nv_bfloat162*>(&uv);
            float2 a0 = __bfloat1622float2(hk[0]), a1 = __bfloat1622float2(hk[1]);
            float2 b0 = __bfloat1622float2(hv[0]), b1 = __bfloat1622float2(hv[1]);
            x[0] = a0.x; x[1] = a0.y; x[2] = a1.x; x[3] = a1.y;
            v4[0] = b0.x; v4[1] = b0.y; v4[2] = b1.x; v4[3] = b1.y;
        } else {
            const float4 fk = *reinterpret_cast<const float4*>(static_cast<const float*>(k_raw) + off);
            const float4 fv = *reinterpret_cast<const float4*>(static_cast<const float*>(v_raw) + off);
            x[0] = fk.x; x[1] = fk.y; x[2] = fk.z; x[3] = fk.w;
            v4[0] = fv.x; v4[1] = fv.y; v4[2] = fv.z; v4[3] = fv.w;
        }
        // cos/sin do not depend on the norm: requested with the row, before the reductions.
        const float4 c = *reinterpret_cast<const float4*>(cosv + (size_t)t * 64 + jr);
        const float4 s = *reinterpret_cast<const float4*>(sinv + (size_t)t * 64 + jr);
        float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float rs = rsqrtf(ss * (1.f / kD) + eps);
        float y[4], partner[4];
#pragma unroll
        for (int e = 0; e < 4; e++) y[e] = x[e] * rs * w4[e];
#pragma unroll
        for (int e = 0; e < 4; e++) partner[e] = __shfl_xor_sync(0xffffffffu, y[e], 16);
        const float c4[4] = {c.x, c.y, c.z, c.w}, s4[4] = {s.x, s.y, s.z, s.w};
        float z[4];
#pragma unroll
        for (int e = 0; e < 4; e++)
            z[e] = lane < 16 ? y[e] * c4[e] - partner[e] * s4[e] : y[e] * c4[e] + partner[e] * s4[e];
        const size_t doff = ((size_t)hh * row_capacity + pos0 + t) * kD + 4 * lane;
        *reinterpret_cast<uint2*>(k_dst + doff) = make_uint2(pack_bf16x2(z[0], z[1]), pack_bf16x2(z[2], z[3]));
        *reinterpret_cast<uint2*>(v_dst + doff) = make_uint2(pack_bf16x2(v4[0], v4[1]), pack_bf16x2(v4[2], v4[3]));
    }
}

// ---- host ---------------------------------------------------------------------------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn()
{
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// Rows [0, rows) of the 8 heads of one layer's BF16 cache as a 3-D tensor {128, rows, 8},
// copied in boxes of {64 dims, box_rows rows, 1 head} with the 128-byte swizzle; rows past
// `rows` read as zeros.
static bool make_rows_map(CUtensorMap* map, const void* base, int rows, int row_capacity, int box_rows)
{
    EncodeTiledFn fn = encode_fn();
    if (!fn || rows <= 0 || box_rows <= 0 || box_rows > 256) return false;
    const cuuint64_t dims[3] = {(cuuint64_t)kD, (cuuint64_t)rows, (cuuint64_t)kHkv};
    const cuuint64_t strides[2] = {(cuuint64_t)kD * 2, (cuuint64_t)row_capacity * kD * 2};
    const cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static bool make_kv_map(CUtensorMap* map, const void* base, int rows, int row_capacity)
{
    return make_rows_map(map, base, rows, row_capacity, kPtKeys);
}

constexpr size_t kPtSmemBytes = 6 * (size_t)kPtTile + 256 + 1024;  // tiles + barriers + alignment slack

}  // namespace tyb

using namespace tyb;

extern "C" int tyb_encode_rows_map(void* map, const void* base, int rows, int row_capacity, int box_rows)
{
    return make_rows_map(static_cast<CUtensorMap*>(map), base, rows, row_capacity, box_rows) ? 0 : 1;
}

extern "C" int tyb_prefill_x_maps(void* const* bases, int world, int max_tokens, void* maps_out)
{
    EncodeTiledFn fn = encode_fn();
    if (!fn || world < 1 || world > 8 || max_tokens <= 0) return (int)cudaErrorInvalidValue;
    CUtensorMap* maps = static_cast<CUtensorMap*>(maps_out);
    memset(maps, 0, sizeof(PrefillPeerMaps));
    const cuuint64_t dims[4] = {(cuuint64_t)kD, (cuuint64_t)kHq, (cuuint64_t)max_tokens, 2};
    const cuuint64_t strides[3] = {(cuuint64_t)kD * 2, (cuuint64_t)kHq * kD * 2, (cuuint64_t)max_tokens * kHq * kD * 2};
    const cuuint32_t box[4] = {64, 1, (cuuint32_t)(max_tokens < kPtRows ? max_tokens : kPtRows), 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    for (int p = 0; p < world; p++) {
        void* slots = static_cast<unsigned char*>(bases[p]) + TYB_PX_HEADER_BYTES;
        if (fn(&maps[p], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, slots, dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return (int)cudaErrorInvalidValue;
    }
    return 0;
}

extern "C" int tyb_kv_prep_launch(const void* k_raw, const void* v_raw, int in_bf16, const float* k_norm,
                                  const float* cos, const float* sin, void* k_dst, void* v_dst, int row_capacity,
                                  int pos0, int S, float eps, int kvh0, int nkvh, void* stream)
{
    if (S <= 0 || nkvh <= 0) return 0;
    const int threads = 256;
    long long blocks = ((long long)S * nkvh + threads / 32 - 1) / (threads / 32);
    if (blocks > 148LL * 16) blocks = 148LL * 16;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)blocks);
    cfg.blockDim = dim3(threads);
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return (int)cudaLaunchKernelEx(&cfg, kv_prep_kernel, k_raw, v_raw, in_bf16, k_norm, cos, sin,
                                   static_cast<__nv_bfloat16*>(k_dst), static_cast<__nv_bfloat16*>(v_dst), row_capacity,
                                   pos0, S, eps, kvh0, nkvh);
}

extern "C" int tyb_prefill_tc_launch(const void* q, int q_bf16, const float* q_norm, const float* cos,
                                     const float* sin, const void* k_cache, const void* v_cache, int row_capacity,
                                     void* out, int out_bf16, int Sq, int pos_offset, float scale, float eps,
                                     int kvh0, int nkvh, int out_head_major, const tyb_prefill_x* xchg_dev,
                                     const void* xchg_maps, unsigned int epoch, void* stream)
{
    if (Sq <= 0 || nkvh <= 0) return 0;
    if (xchg_dev && !xchg_maps) return (int)cudaErrorInvalidValue;
    // Once per device: the shared-memory opt-in, and a check that the kernel was compiled
    // for the launch register count its setmaxnreg split is sized against (a split above
    // the launch's registers would never be granted).
    static bool ready[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= 64) return (int)cudaErrorInvalidDevice;
    if (!ready[dev]) {
        cudaFuncAttributes fa;
        e = cudaFuncGetAttributes(&fa, prefill_tc_kernel);
        if (e != cudaSuccess) return (int)e;
        if (fa.numRegs != kPtLaunchRegs || fa.maxThreadsPerBlock < kPtThreads) return (int)cudaErrorInvalidConfiguration;
        e = cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPtSmemBytes);
        if (e != cudaSuccess) return (int)e;
        ready[dev] = true;
    }
    PrefillTcArgs a;
    a.q = q;
    a.q_bf16 = q_bf16;
    a.q_norm = q_norm;
    a.cos = cos;
    a.sin = sin;
    a.out = out;
    a.out_bf16 = out_bf16;
    a.Sq = Sq;
    a.pos_offset = pos_offset;
    a.total_kv = pos_offset + Sq;
    a.n_qtiles = (Sq + kPtRows - 1) / kPtRows;
    a.scale_log2 = scale * kLog2e;
    a.eps = eps;
    a.kvh0 = kvh0;
    a.nkvh = nkvh;
    a.out_head_major = out_head_major;
    a.xchg = xchg_dev;
    a.epoch = epoch;
    a.status = tyb_status_word();
    if (!a.status) return (int)cudaErrorInvalidSymbol;
    a.mirror = tyb_status_mirror_device();
    a.wait_ns = tyb_wait_limit();
    CUtensorMap mk, mv;
    if (!make_kv_map(&mk, k_cache, a.total_kv, row_capacity) || !make_kv_map(&mv, v_cache, a.total_kv, row_capacity))
        return (int)cudaErrorInvalidValue;
    // Programmatic dependent launch: the CTAs may start (TMEM, barriers, the query prologue) while
    // kv_prep finishes; the TMA producer waits for it before reading the cache rows.  This needs
    // kv_prep to be the previous kernel in the stream, which lets it launch only after all its CTAs
    // have waited for everything before it (so that whatever produced q, q_norm, cos and sin has
    // completed): the only caller launches the two back to back.  The outputs are written after
    // the wait (the epilogue follows the P.V of every tile, which follows the K/V loads).
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(a.n_qtiles * nkvh));
    cfg.blockDim = dim3(kPtThreads);
    cfg.dynamicSmemBytes = kPtSmemBytes;
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    PrefillPeerMaps px;
    if (xchg_maps)
        memcpy(&px, xchg_maps, sizeof px);
    else
        memset(&px, 0, sizeof px);
    return (int)cudaLaunchKernelEx(&cfg, prefill_tc_kernel, mk, mv, a, px);
}
