// Asynchronous-copy and mbarrier helpers (inline PTX, sm_100a).
//
// Every wait is bounded by %globaltimer: a kernel that does not see its
// barrier complete within FB_WAIT_LIMIT_NS records an error code in its
// translation unit's device status word and bails out, so a lost arrival can
// never hang the GPU.
#pragma once

#include <cstdint>

#ifndef FB_WAIT_LIMIT_NS
#define FB_WAIT_LIMIT_NS 2000000000ull
#endif

namespace fb {

// Device status codes written on a bounded-wait timeout.
enum DeviceStatus : uint32_t {
    DEV_OK = 0,
    DEV_ROWS_WAIT_TIMEOUT = 1,
    DEV_GEMM_PRODUCER_TIMEOUT = 2,
    DEV_GEMM_MMA_TIMEOUT = 3,
    DEV_GEMM_EPILOGUE_TIMEOUT = 4,
    DEV_ATTN_TIMEOUT = 5,
    DEV_SELFTEST_TIMEOUT = 6,  // fb_selftest_bounded_wait: the wait gave up as intended
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Makes barrier initialisation visible to the async proxy (TMA, tcgen05).
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's generic-proxy shared-memory accesses before later
// async-proxy accesses (a TMA overwriting a buffer that was just read).
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
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

// Waits for the barrier phase with the given parity to complete.  Returns
// false if it did not within `limit_ns` nanoseconds.
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity))
        if (globaltimer_ns() - t0 > limit_ns) return false;
    return true;
}

// The bounded wait every kernel uses: FB_WAIT_LIMIT_NS.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    return mbar_wait_for(bar, parity, FB_WAIT_LIMIT_NS);
}

// Bulk (non-tensor) copy global -> shared, completing on `bar` with `bytes`
// of transaction count.  Addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

}  // namespace fb
