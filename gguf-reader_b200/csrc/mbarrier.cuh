// mbarrier.cuh -- mbarrier waits and 1-D bulk copies (global -> shared) shared
// by the GEMV and attention kernels.  Every wait is bounded: on expiry the
// caller's error flags get ERRF_TIMEOUT and the wait returns false.
#pragma once
#include "common.cuh"

namespace ggc {

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

constexpr uint32_t BULK_WAIT_LIMIT = 1u << 16;   // x up to 20 us suspend each: ~1.3 s bound

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 20000;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait on phase `parity`; false (and ERRF_TIMEOUT) when the limit expires.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* errf) {
    for (uint32_t i = 0; i < BULK_WAIT_LIMIT; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    if (errf) atomicExch(&errf[ERRF_TIMEOUT], 1);
    return false;
}
// 1-D bulk copy global -> shared, completion counted on `bar` (no multicast)
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}

// orders this thread's earlier generic-proxy shared-memory accesses before
// later bulk copies into the same bytes
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

}  // namespace ggc
