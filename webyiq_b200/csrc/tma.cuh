// Shared-memory barriers, TMA copies and the device error word's codes, shared by
// the tensor-core kernels.  No copy here uses cluster multicast.
#pragma once

#include <cstdint>

namespace w4a8 {

constexpr long long kWaitLimitCycles = 1ll << 29;  // bounded waits: ~0.3 s at 2 GHz

// Bits of the device error word (set by a kernel whose bounded wait gave up).
enum : unsigned int {
    DEV_ERR_TMA_TIMEOUT = 1u,   // GEMV: a weight copy never landed
    DEV_ERR_GEMM_TIMEOUT = 2u,  // GEMM: a pipeline wait gave up
    DEV_ERR_SELFTEST = 4u,      // w4a8_selftest_wait_timeout: its wait gave up (as it must)
    DEV_ERR_XCHG_TIMEOUT = 8u,  // peer key exchange: a rank's flag never arrived
};

// --- TMA bulk copies and mbarriers (no cluster multicast anywhere) -----------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// Orders this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (TMA) accesses.
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tma_bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
// 16-byte copies global -> shared issued by this thread (LDGSTS), in commit groups.
// Kernels launched with programmatic dependent launch use these for data they fetch
// before griddepcontrol.wait, and each thread waits for its own groups with
// cp_async_wait_upto before it blocks there: bulk copies a dependent grid issues
// before the wait complete only once the previous grid has finished, and so do
// completions that a thread parked in the wait would signal to an mbarrier.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// Wait until at most n (0..2) of this thread's newest commit groups are pending.
__device__ __forceinline__ void cp_async_wait_upto(int n) {
    if (n <= 0)
        asm volatile("cp.async.wait_group 0;" ::: "memory");
    else if (n == 1)
        asm volatile("cp.async.wait_group 1;" ::: "memory");
    else
        asm volatile("cp.async.wait_group 2;" ::: "memory");
}
// Whether phase `parity` of the barrier has completed (one non-blocking test).
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}
// Wait for phase `parity` of the barrier, giving up after kWaitLimitCycles: a
// non-blocking test first (the phase is usually complete by now), then the
// hardware-suspending try_wait, so a waiting thread does not spin on the issue port.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t a = smem_u32(bar);
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
    const long long t0 = clock64();
    while (true) {
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
        if (clock64() - t0 > kWaitLimitCycles) return false;
    }
}

}  // namespace w4a8
