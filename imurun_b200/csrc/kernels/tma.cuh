// tma.cuh — mbarriers and bulk (TMA) copies from global to shared memory.
//
// Every wait is bounded: it gives up after kWaitNs of device time (or once
// another thread raised the CTA's abort flag), so a lost transfer ends the
// kernel with an error flag instead of hanging the GPU.
#pragma once

#include <stdint.h>

namespace fb {

constexpr long long kWaitNs = 2000000000LL;   // 2 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// try_wait with a suspend-time hint: the thread is parked (not spinning, so it
// takes no issue slots from the warps that do work) until the phase completes
// or about kSuspendNs pass.
constexpr uint32_t kSuspendNs = 2000;
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendNs)
        : "memory");
    return ok != 0;
}
// Bounded wait: false after kWaitNs or once another thread raised *abort.
// The clock is read only once the first try has failed; t_start (optional)
// receives that time when the wait gives up.
// waited (optional) accumulates the ns spent when the first try failed.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          unsigned long long* t_start = nullptr, unsigned long long* waited = nullptr) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = gtimer();
    for (unsigned i = 1;; ++i) {
        if (mbar_try_wait_sleep(bar, parity)) {
            if (waited) *waited += gtimer() - t0;
            return true;
        }
        if ((i & 7) == 0 && (*abort || (long long)(gtimer() - t0) > kWaitNs)) {
            if (t_start) *t_start = t0;
            return false;
        }
    }
}
// Bounded wait that ignores the abort flag (used while draining).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    const unsigned long long t0 = gtimer();
    for (unsigned i = 0;; ++i) {
        if (mbar_try_wait_sleep(bar, parity)) return true;
        if ((i & 7) == 7 && (long long)(gtimer() - t0) > kWaitNs) return false;
    }
}
// One bulk copy global -> shared (both 16-byte aligned, bytes % 16 == 0),
// completing `bytes` of the barrier's transaction count.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

}  // namespace fb
