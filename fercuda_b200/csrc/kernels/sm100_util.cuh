// Small sm_100a helpers shared by the kernels: mbarriers with bounded waits,
// 1-D bulk (TMA) copies global -> shared, proxy fences, error reporting.
#pragma once

#include <cstdint>

namespace fer::dev {

// Error bits written (atomicOr) into the caller's error word.
enum : uint32_t {
    kErrTimeoutLoad = 1u << 0,   // a bulk copy did not land within the wait limit
    kErrTimeoutMma = 1u << 1,    // a tensor-core commit did not arrive in time
    kErrBadShape = 1u << 2,      // launched with a shape the kernel cannot take
    kErrTimeoutSync = 1u << 3,   // a producer/consumer handshake timed out
};

// About one second at B200 clocks.
constexpr long long kWaitCycles = 2000000000ll;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Fetches a TMA tensor map (a __grid_constant__ kernel parameter) into the
// descriptor cache ahead of its first use, so the first tensor copy does not
// wait for it. It reads only kernel parameters: safe before a programmatic
// launch wait.
__device__ __forceinline__ void prefetch_tmap(const void* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait that lets the hardware suspend the thread for up to `ns`
// nanoseconds while the phase is incomplete.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(ns)
        : "memory");
    return ok != 0;
}

// Waits for the phase with the given parity to complete; false after about
// one second (the caller reports the error and stops). Threads sleep in
// try_wait between polls and read the clock only every 64 polls, so waiting
// warps take almost no issue slots from working ones.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (uint32_t k = 1;; ++k) {
        if (mbar_try_wait_sleep(bar, parity, 2000)) return true;
        if ((k & 63u) == 0 && clock64() - t0 > kWaitCycles) return false;
    }
}

// 1-D bulk copy global -> shared, completion counted on `bar` in bytes.
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// Orders this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (bulk copy / tensor core) accesses.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// A shared flag read by a whole warp, agreed across its lanes (any lane that
// sees it set makes it set for all), so the warp takes one branch.
__device__ __forceinline__ bool warp_flag(volatile int* f) { return __any_sync(0xffffffffu, *f != 0); }

__device__ __forceinline__ void report(uint32_t* err, uint32_t bits) {
    if (err) atomicOr(err, bits);
}

__device__ __forceinline__ void st_global_cs(float* p, float v) {
    asm volatile("st.global.cs.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

}  // namespace fer::dev
