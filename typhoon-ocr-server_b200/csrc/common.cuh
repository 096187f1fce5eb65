// common.cuh -- device helpers shared by the sm_100a kernels of the GQA attention path.
//
// Model constants are those of the Qwen3-VL-2B text decoder the reference serves
// (kernel/attention.c:43-46): 16 query heads, 8 KV heads, head_dim 128, GQA group 2
// (query head h reads KV head h/2, kernel/attention.c:170).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "attn_shim.h"

namespace tyb {

constexpr int kHq = 16;
constexpr int kHkv = 8;
constexpr int kD = 128;
constexpr int kGroup = 2;
constexpr float kLog2e = 1.4426950408889634f;

// Status word shared by every kernel of this library.  Kernels never trap: a wait
// that runs out of time or an index that fails a check sets a bit here and the
// kernel returns; the host reads it back (attn_sync, synchronous entry points).
// Relocatable translation units name the symbol; a whole-program one (TYB_WHOLE_PROGRAM)
// receives its address (tyb_status_word) as a kernel argument.
//
// A raised bit also flags a page-locked host word (the mirror, NULL until the host sets it
// up), so that a blocking call learns that nothing went wrong from a stream synchronisation
// alone and reads the status word back only when the mirror is set.
#ifndef TYB_WHOLE_PROGRAM
extern __device__ unsigned int g_status;
extern __device__ unsigned int* g_status_mirror;

__device__ __forceinline__ void flag_mirror(unsigned int* mirror)
{
    if (mirror) *reinterpret_cast<volatile unsigned int*>(mirror) = 1u;
}

__device__ __forceinline__ void raise_status(unsigned int bits)
{
    atomicOr(&g_status, bits);
    flag_mirror(g_status_mirror);
}
#else
__device__ __forceinline__ void flag_mirror(unsigned int* mirror)
{
    if (mirror) *reinterpret_cast<volatile unsigned int*>(mirror) = 1u;
}
#endif

__device__ __forceinline__ uint64_t globaltimer_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---- element conversions -------------------------------------------------------------
__device__ __forceinline__ void load8(const float* p, float (&x)[8])
{
    float4 a = *reinterpret_cast<const float4*>(p);
    float4 b = *reinterpret_cast<const float4*>(p + 4);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&x)[8])
{
    uint4 u = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        float2 f = __bfloat1622float2(h[i]);
        x[2 * i] = f.x;
        x[2 * i + 1] = f.y;
    }
}

__device__ __forceinline__ void store8(float* p, const float (&x)[8])
{
    *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(x[4], x[5], x[6], x[7]);
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&x)[8])
{
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; i++) h[i] = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = u;
}

// ---- mbarrier + bulk async copy (TMA, non-tensor form) -------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Arrive on an mbarrier without a transaction count (completes a phase with no copy).
__device__ __forceinline__ void mbar_arrive(uint64_t* bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// try_wait that may suspend the thread in hardware for up to `hint_ns` before reporting
// "not yet" (the thread stops competing for issue slots while it waits).
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Wait for phase `parity` of an mbarrier, giving up after `limit_ns` of wall time.
// Returns false (and sets `status_bit` in *status) when the limit ran out.
__device__ __forceinline__ bool mbar_wait_bounded_to(uint64_t* bar, uint32_t parity, uint64_t limit_ns,
                                                     unsigned int status_bit, unsigned int* status,
                                                     unsigned int* mirror)
{
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait_sleep(bar, parity, 2000u)) return true;
        if (globaltimer_ns() - t0 > limit_ns) {
            atomicOr(status, status_bit);
            flag_mirror(mirror);
            return false;
        }
    }
}

// Non-blocking test of phase `parity`.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Like mbar_wait_bounded_to, but polling without suspending: for a single latency-critical
// thread (it reacts within a few cycles of the phase completing, at the price of issue slots).
__device__ __forceinline__ bool mbar_spin_bounded_to(uint64_t* bar, uint32_t parity, uint64_t limit_ns,
                                                     unsigned int status_bit, unsigned int* status,
                                                     unsigned int* mirror)
{
    if (mbar_test_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t n = 1;; n++) {
        if (mbar_test_wait(bar, parity)) return true;
        if ((n & 255u) == 0 && globaltimer_ns() - t0 > limit_ns) {
            atomicOr(status, status_bit);
            flag_mirror(mirror);
            return false;
        }
    }
}

#ifndef TYB_WHOLE_PROGRAM
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint64_t limit_ns, unsigned int status_bit)
{
    return mbar_wait_bounded_to(bar, parity, limit_ns, status_bit, &g_status, g_status_mirror);
}

// The current wait limit of this device (attn_set_wait_limit_ns; kWaitLimitNs until set).
// Whole-program translation units receive it as a kernel argument instead.
extern __device__ unsigned long long g_wait_limit_ns;
__device__ __forceinline__ uint64_t wait_limit_ns() { return g_wait_limit_ns; }
#endif

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`.
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                         uint64_t* bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Bulk prefetch of global memory into L2 (no shared memory, no completion to wait for).
// Address 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void* gmem, uint32_t bytes)
{
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(gmem), "r"(bytes) : "memory");
}

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // default limit, 2 s: far beyond any legitimate wait

}  // namespace tyb
