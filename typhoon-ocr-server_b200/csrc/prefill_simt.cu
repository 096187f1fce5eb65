// prefill_simt.cu -- FP32 causal GQA flash attention on CUDA cores.
//
// The exact-FP32 path behind the drop-in entry points attention_prefill_gqa and
// attention_chunked_prefill_gqa, whose inputs are FP32 and whose parity bar against the
// reference (kernel/attention.c:252-381 and :413-543) is max-abs 2e-3 / rel-L2 1e-3.
// FP32 has no tensor-core form on sm_100a (tf32 keeps 10 mantissa bits), so this
// kernel keeps full FP32 products and sums; the BF16 tensor-core kernel is the
// throughput path.
//
// One CTA = 32 query tokens x the 2 query heads of one KV head (64 rows, GQA folded into
// the tile) against 64-key tiles of that KV head, online softmax in base 2.
// Thread (rg = tid/16, cg = tid%16) owns rows 4rg..4rg+3; in QK^T it owns keys
// cg + 16j (j < 4), in PV it owns dims 4cg..4cg+3 and 64+4cg..64+4cg+3.  A row's 16
// owners are one half-warp, so row max/sum reduce with four xor-shuffles.
#include "common.cuh"

namespace tyb {

constexpr int kPfThreads = 256;
constexpr int kPfTok = 32;             // query tokens per CTA
constexpr int kPfRows = kPfTok * kGroup;  // 64 rows: row r = head (r / 32), token (r % 32)
constexpr int kPfKeys = 64;
constexpr int kQkPad = kD + 4;         // padded row: 16-byte column reads hit distinct banks
constexpr int kPPad = kPfKeys + 4;

struct PrefillSimtArgs {
    const float* q;
    float* out;
    const void* k;
    const void* v;
    long long row_stride;
    long long head_stride;
    int Sq;
    int Sk;
    int pos_offset;
    float scale_log2;
};

__device__ __forceinline__ float exp2_approx(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float4 load4_as_f32(const float* p) { return *reinterpret_cast<const float4*>(p); }

__device__ __forceinline__ float4 load4_as_f32(const __nv_bfloat16* p)
{
    uint2 u = *reinterpret_cast<const uint2*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
    return make_float4(a.x, a.y, b.x, b.y);
}

template <typename TKV>
__global__ void __launch_bounds__(kPfThreads) prefill_simt_kernel(const PrefillSimtArgs a)
{
    extern __shared__ __align__(16) float sm[];
    float* Qs = sm;                        // [64][132]
    float* Ks = Qs + kPfRows * kQkPad;     // [64][132]
    float* Vs = Ks + kPfKeys * kQkPad;     // [64][128]
    float* Ps = Vs + kPfKeys * kD;         // [64][68]

    const int ntq = (a.Sq + kPfTok - 1) / kPfTok;
    const int qt = ntq - 1 - (int)blockIdx.x;  // longest tiles first
    const int kvh = blockIdx.y;
    const int q0 = qt * kPfTok;
    const int ntok = min(kPfTok, a.Sq - q0);
    const int tid = threadIdx.x;
    const int rg = tid >> 4;
    const int cg = tid & 15;
    const TKV* Kg = static_cast<const TKV*>(a.k) + (size_t)kvh * a.head_stride;
    const TKV* Vg = static_cast<const TKV*>(a.v) + (size_t)kvh * a.head_stride;

    // Q tile: rows r -> token q0 + r%32, head 2*kvh + r/32 (zeros past Sq).
    for (int idx = tid; idx < kPfRows * (kD / 4); idx += kPfThreads) {
        const int r = idx / (kD / 4), c4 = idx % (kD / 4);
        const int tok = r & (kPfTok - 1), g = r >> 5;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (tok < ntok)
            v = *reinterpret_cast<const float4*>(a.q + (size_t)(q0 + tok) * (kHq * kD) +
                                                 (size_t)(kGroup * kvh + g) * kD + 4 * c4);
        *reinterpret_cast<float4*>(Qs + r * kQkPad + 4 * c4) = v;
    }

    float m_run[4], l_run[4], o[4][8];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        m_run[i] = -INFINITY;
        l_run[i] = 0.f;
#pragma unroll
        for (int j = 0; j < 8; j++) o[i][j] = 0.f;
    }
    int qpos[4];
#pragma unroll
    for (int i = 0; i < 4; i++) qpos[i] = a.pos_offset + q0 + ((4 * rg + i) & (kPfTok - 1));

    const int kv_end = min(a.Sk, a.pos_offset + q0 + ntok);
    for (int kv0 = 0; kv0 < kv_end; kv0 += kPfKeys) {
        __syncthreads();  // previous tile fully consumed
        for (int idx = tid; idx < kPfKeys * (kD / 4); idx += kPfThreads) {
            const int r = idx / (kD / 4), c4 = idx % (kD / 4);
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (kv0 + r < kv_end) {
                const size_t off = (size_t)(kv0 + r) * a.row_stride + 4 * c4;
                kv = load4_as_f32(Kg + off);
                vv = load4_as_f32(Vg + off);
            }
            *reinterpret_cast<float4*>(Ks + r * kQkPad + 4 * c4) = kv;
            *reinterpret_cast<float4*>(Vs + r * kD + 4 * c4) = vv;
        }
        __syncthreads();

        float s[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) s[i][j] = 0.f;
#pragma unroll 4
        for (int d = 0; d < kD; d += 4) {
            float4 qa[4], kb[4];
#pragma unroll
            for (int i = 0; i < 4; i++) qa[i] = *reinterpret_cast<const float4*>(Qs + (4 * rg + i) * kQkPad + d);
#pragma unroll
            for (int j = 0; j < 4; j++) kb[j] = *reinterpret_cast<const float4*>(Ks + (cg + 16 * j) * kQkPad + d);
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    s[i][j] = fmaf(qa[i].x, kb[j].x, s[i][j]);
                    s[i][j] = fmaf(qa[i].y, kb[j].y, s[i][j]);
                    s[i][j] = fmaf(qa[i].z, kb[j].z, s[i][j]);
                    s[i][j] = fmaf(qa[i].w, kb[j].w, s[i][j]);
                }
        }

        float alpha[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float mt = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int kp = kv0 + cg + 16 * j;
                s[i][j] = (kp <= qpos[i] && kp < kv_end) ? s[i][j] * a.scale_log2 : -INFINITY;
                mt = fmaxf(mt, s[i][j]);
            }
#pragma unroll
            for (int off = 8; off >= 1; off >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
            const float m_new = fmaxf(m_run[i], mt);
            if (m_new == -INFINITY) {  // row has seen no visible key yet
                alpha[i] = 1.f;
#pragma unroll
                for (int j = 0; j < 4; j++) s[i][j] = 0.f;
            } else {
                alpha[i] = exp2_approx(m_run[i] - m_new);  // exp2(-inf) = 0 on the first hit
#pragma unroll
                for (int j = 0; j < 4; j++) s[i][j] = exp2_approx(s[i][j] - m_new);
            }
            m_run[i] = m_new;
            float ls = 0.f;
#pragma unroll
            for (int j = 0; j < 4; j++) ls += s[i][j];
            l_run[i] = l_run[i] * alpha[i] + ls;
#pragma unroll
            for (int j = 0; j < 4; j++) Ps[(4 * rg + i) * kPPad + cg + 16 * j] = s[i][j];
#pragma unroll
            for (int j = 0; j < 8; j++) o[i][j] *= alpha[i];
        }
        __syncthreads();

#pragma unroll 4
        for (int key = 0; key < kPfKeys; key++) {
            const float4 va = *reinterpret_cast<const float4*>(Vs + key * kD + 4 * cg);
            const float4 vb = *reinterpret_cast<const float4*>(Vs + key * kD + 64 + 4 * cg);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float p = Ps[(4 * rg + i) * kPPad + key];
                o[i][0] = fmaf(p, va.x, o[i][0]);
                o[i][1] = fmaf(p, va.y, o[i][1]);
                o[i][2] = fmaf(p, va.z, o[i][2]);
                o[i][3] = fmaf(p, va.w, o[i][3]);
                o[i][4] = fmaf(p, vb.x, o[i][4]);
                o[i][5] = fmaf(p, vb.y, o[i][5]);
                o[i][6] = fmaf(p, vb.z, o[i][6]);
                o[i][7] = fmaf(p, vb.w, o[i][7]);
            }
        }
    }

#pragma unroll
    for (int i = 0; i < 4; i++) {
        float l = l_run[i];
#pragma unroll
        for (int off = 8; off >= 1; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
        const int r = 4 * rg + i;
        const int tok = r & (kPfTok - 1), g = r >> 5;
        if (tok >= ntok) continue;
        const float inv = l > 0.f ? 1.f / l : 0.f;  // rows with no visible key give 0 (:348)
        float* dst = a.out + (size_t)(q0 + tok) * (kHq * kD) + (size_t)(kGroup * kvh + g) * kD;
        *reinterpret_cast<float4*>(dst + 4 * cg) =
            make_float4(o[i][0] * inv, o[i][1] * inv, o[i][2] * inv, o[i][3] * inv);
        *reinterpret_cast<float4*>(dst + 64 + 4 * cg) =
            make_float4(o[i][4] * inv, o[i][5] * inv, o[i][6] * inv, o[i][7] * inv);
    }
}

constexpr size_t kPfSmemBytes =
    sizeof(float) * ((size_t)kPfRows * kQkPad + (size_t)kPfKeys * kQkPad + (size_t)kPfKeys * kD +
                     (size_t)kPfRows * kPPad);

template <typename TKV>
static int launch_prefill_simt(const PrefillSimtArgs& a, void* stream)
{
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(prefill_simt_kernel<TKV>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPfSmemBytes);
        if (e != cudaSuccess) return (int)e;
        attr_set = true;
    }
    dim3 grid((a.Sq + kPfTok - 1) / kPfTok, kHkv);
    prefill_simt_kernel<TKV><<<grid, kPfThreads, kPfSmemBytes, (cudaStream_t)stream>>>(a);
    return (int)cudaGetLastError();
}

}  // namespace tyb

using namespace tyb;

extern "C" int tyb_prefill_simt_launch(const float* q, float* out, const void* k, const void* v,
                                       long long row_stride, long long head_stride, int kv_dtype,
                                       int Sq, int Sk, int pos_offset, float scale, void* stream)
{
    if (Sq <= 0) return 0;
    PrefillSimtArgs a;
    a.q = q;
    a.out = out;
    a.k = k;
    a.v = v;
    a.row_stride = row_stride;
    a.head_stride = head_stride;
    a.Sq = Sq;
    a.Sk = Sk;
    a.pos_offset = pos_offset;
    a.scale_log2 = scale * kLog2e;
    if (kv_dtype == TYB_BF16) return launch_prefill_simt<__nv_bfloat16>(a, stream);
    return launch_prefill_simt<float>(a, stream);
}
