// kv_write.cu -- KV-cache row writes and the library status word.
//
// kv_cache_append (kernel/kv_cache.c:53-65) and kv_cache_append_prefill (:80-104) copy
// token-major K/V rows [S][8][128] into the head-first cache [8][max_seq][128] of one
// layer at rows seq_len.. .  On the device that is one scatter kernel: thread t moves
// 8 contiguous elements (one 16-byte load per 4 fp32 values, one 16-byte store of bf16
// or two of fp32), converting to the cache's element type on the way.
#include "common.cuh"

namespace tyb {

__device__ unsigned int g_status = 0u;
__device__ unsigned int* g_status_mirror = nullptr;
__device__ unsigned long long g_wait_limit_ns = kWaitLimitNs;

static_assert(kD / 8 == 16 && kHkv == 8, "kv_scatter_kernel's index shifts");

template <typename TDst>
__global__ void kv_scatter_kernel(const float* __restrict__ k_src, const float* __restrict__ v_src,
                                  TDst* __restrict__ k_dst, TDst* __restrict__ v_dst,
                                  int row_capacity, int pos0, int S)
{
    // One thread per (tensor, token, head, 8-element group): 2 * S * 8 * 16 threads (< 2^27: 32-bit
    // indices, the division by S once per element group).
    const int n = 2 * S * kHkv * (kD / 8);
    for (int i = (int)(blockIdx.x * blockDim.x + threadIdx.x); i < n; i += (int)(gridDim.x * blockDim.x)) {
        const int c = i & (kD / 8 - 1);
        const int th = i >> 4;  // i / (kD / 8)
        const int h = th & (kHkv - 1);
        const int tt = th >> 3;  // th / kHkv
        const int which = tt >= S;
        const int t = tt - which * S;
        const float* src = (which ? v_src : k_src) + ((size_t)t * kHkv + h) * kD + 8 * c;
        TDst* dst = (which ? v_dst : k_dst) + ((size_t)h * row_capacity + pos0 + t) * kD + 8 * c;
        float x[8];
        load8(src, x);
        store8(dst, x);
    }
}

}  // namespace tyb

using namespace tyb;

extern "C" int tyb_kv_scatter_launch(const float* k_src, const float* v_src, void* k_dst,
                                     void* v_dst, int row_capacity, int pos0, int S, int kv_dtype,
                                     void* stream)
{
    if (S <= 0) return 0;
    const long long n = 2LL * S * kHkv * (kD / 8);
    if (n >= (1LL << 31)) return (int)cudaErrorInvalidValue;
    const int threads = 256;
    long long blocks = (n + threads - 1) / threads;
    if (blocks > 148LL * 16) blocks = 148LL * 16;
    if (kv_dtype == TYB_BF16)
        kv_scatter_kernel<__nv_bfloat16><<<(unsigned)blocks, threads, 0, (cudaStream_t)stream>>>(
            k_src, v_src, static_cast<__nv_bfloat16*>(k_dst), static_cast<__nv_bfloat16*>(v_dst),
            row_capacity, pos0, S);
    else
        kv_scatter_kernel<float><<<(unsigned)blocks, threads, 0, (cudaStream_t)stream>>>(
            k_src, v_src, static_cast<float*>(k_dst), static_cast<float*>(v_dst), row_capacity,
            pos0, S);
    return (int)cudaGetLastError();
}

// The status mirror: one page-locked, device-mapped host word for the process, its device
// address stored in g_status_mirror on each device once (tyb_status_mirror_setup, called
// where caches are allocated).  Until then kernels flag nothing and the host always reads
// the status word back.
static unsigned int* g_mirror_host = nullptr;
static unsigned int* g_mirror_dev[64];
static bool g_mirror_ready[64];

extern "C" int tyb_status_mirror_setup(void)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= 64) return (int)cudaErrorInvalidDevice;
    if (g_mirror_ready[dev]) return 0;
    if (!g_mirror_host) {
        void* p = nullptr;
        e = cudaHostAlloc(&p, sizeof(unsigned int), cudaHostAllocMapped | cudaHostAllocPortable);
        if (e != cudaSuccess) return (int)e;
        g_mirror_host = static_cast<unsigned int*>(p);
        *g_mirror_host = 0u;
    }
    void* d = nullptr;
    e = cudaHostGetDevicePointer(&d, g_mirror_host, 0);
    if (e != cudaSuccess) return (int)e;
    unsigned int* dp = static_cast<unsigned int*>(d);
    e = cudaMemcpyToSymbol(g_status_mirror, &dp, sizeof dp);
    if (e != cudaSuccess) return (int)e;
    g_mirror_dev[dev] = dp;
    g_mirror_ready[dev] = true;
    return 0;
}

extern "C" unsigned int* tyb_status_mirror_host(void)
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || !g_mirror_ready[dev]) return nullptr;
    return g_mirror_host;
}

extern "C" unsigned int* tyb_status_mirror_device(void)
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || !g_mirror_ready[dev]) return nullptr;
    return g_mirror_dev[dev];
}

// Head-major [16][S][128] -> token-major [S][16][128]: one 16-byte vector per thread step.
__global__ void heads_to_tokens_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, int S, int vec_per_row)
{
    const long long total = (long long)kHq * S * vec_per_row;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int v = (int)(i % vec_per_row);
        const long long hr = i / vec_per_row;  // h * S + t
        const int t = (int)(hr % S), h = (int)(hr / S);
        dst[((long long)t * kHq + h) * vec_per_row + v] = src[i];
    }
}

extern "C" int tyb_heads_to_tokens_launch(const void* src, void* dst, int S, int elem_bytes, void* stream)
{
    if (S <= 0) return 0;
    const int vec_per_row = kD * elem_bytes / 16;
    const long long total = (long long)kHq * S * vec_per_row;
    long long blocks = (total + 255) / 256;
    if (blocks > 148LL * 32) blocks = 148LL * 32;
    heads_to_tokens_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(static_cast<const uint4*>(src),
                                                                               static_cast<uint4*>(dst), S, vec_per_row);
    return (int)cudaGetLastError();
}

extern "C" unsigned int* tyb_status_word(void)
{
    // Device address of the status word on the current device (looked up once per device).
    static unsigned int* addr[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    if (!addr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_status) != cudaSuccess) return nullptr;
        addr[dev] = static_cast<unsigned int*>(p);
    }
    return addr[dev];
}

extern "C" int tyb_status_fetch(unsigned int* bits, void* stream)
{
    // One pinned word per process receives the status copy, so the read is queued behind
    // the caller's work and a single stream synchronisation covers both.
    static unsigned int* pinned = nullptr;
    if (!pinned) {
        cudaError_t e = cudaHostAlloc(reinterpret_cast<void**>(&pinned), sizeof(unsigned int), cudaHostAllocDefault);
        if (e != cudaSuccess) {
            pinned = nullptr;
            return (int)e;
        }
    }
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e = cudaMemcpyFromSymbolAsync(pinned, g_status, sizeof(unsigned int), 0, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return (int)e;
    *bits = *pinned;
    if (*bits) {
        const unsigned int zero = 0u;
        e = cudaMemcpyToSymbol(g_status, &zero, sizeof zero);
    }
    return (int)e;
}

// Wait limit of the bounded waits, per device: the device variable the relocatable kernels read,
// and a host copy the launchers of the whole-program kernels pass as an argument.
static unsigned long long g_wait_limit_host[64];

extern "C" int tyb_set_wait_limit(unsigned long long ns)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= 64) return (int)cudaErrorInvalidDevice;
    e = cudaMemcpyToSymbol(g_wait_limit_ns, &ns, sizeof ns);
    if (e != cudaSuccess) return (int)e;
    g_wait_limit_host[dev] = ns;
    return 0;
}

extern "C" unsigned long long tyb_wait_limit(void)
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || !g_wait_limit_host[dev]) return kWaitLimitNs;
    return g_wait_limit_host[dev];
}
