// mbarrier and bulk-copy helpers shared by the staged kernels.  Every wait is bounded in time:
// after kWaitLimitNs it gives up and reports failure, so a kernel never spins forever.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace draco {
namespace sync {

constexpr uint64_t kWaitLimitNs = 2000000000ull;   // 2 s
// try_wait may suspend the polling thread up to this long (0: poll with test_wait)
#ifndef DRACO_MBAR_SUSPEND_NS
#define DRACO_MBAR_SUSPEND_NS 1000
#endif
constexpr uint32_t kSuspendNs = DRACO_MBAR_SUSPEND_NS;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    if (kSuspendNs == 0)
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(smem_addr(bar)), "r"(parity)
            : "memory");
    else
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(smem_addr(bar)), "r"(parity), "r"(kSuspendNs)
            : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// bounded wait for the phase with the given parity; false after kWaitLimitNs
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1;; i++) {
        if (mbar_try(bar, parity)) return true;
        if ((i & 63) == 0 && global_ns() - t0 > kWaitLimitNs) return false;
    }
}
// orders this thread's earlier generic-proxy accesses of shared memory before its later
// async-proxy ones (a bulk copy into a buffer that was just read)
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// global -> shared bulk copy (both addresses 16-byte aligned, bytes a multiple of 16), completing
// on bar's transaction count
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

}  // namespace sync
}  // namespace draco
