// tma.cuh -- 1D bulk copies (TMA) from global into shared memory, completed
// on an mbarrier, for kernels that stage a block's inputs in one go.
// No multicast: every copy reads this GPU's own memory into this CTA.
#pragma once
#include <cuda_runtime.h>

namespace msp {

// mbarrier polls before a wait gives up (each poll may suspend the thread
// for a while in hardware, so this is seconds, far beyond any real copy).
constexpr unsigned kBulkSpinLimit = 1u << 22;

__device__ __forceinline__ unsigned smem_addr(const void* p)
{
    return (unsigned)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(unsigned long long* bar)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"(smem_addr(bar)) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(unsigned long long* bar, unsigned bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                 :: "r"(smem_addr(bar)), "r"(bytes) : "memory");
}

// dst, src and bytes must all be multiples of 16 bytes.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, unsigned bytes,
                                          unsigned long long* bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        :: "r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(unsigned long long* bar, unsigned parity)
{
    unsigned ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(smem_addr(bar)), "r"(parity) : "memory");
    return ok != 0;
}

// Waits for phase `parity`; false after kBulkSpinLimit polls.
__device__ __forceinline__ bool mbar_wait_bounded(unsigned long long* bar, unsigned parity)
{
    for (unsigned k = 0; k < kBulkSpinLimit; k++)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

}  // namespace msp
