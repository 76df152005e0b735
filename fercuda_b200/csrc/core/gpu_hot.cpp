// gpu_hot_*: one device pool per runtime, carved by the TLSF allocator.
//
// Replaces the pool part of the reference GPU hot runtime:
//   init + pool sizing      native/core/runtime/modules/hot_runtime_init.inl:8-364
//   default config          native/core/runtime/modules/hot_runtime_prelude.inl:471-505
//   alloc / free / async    native/core/runtime/modules/hot_runtime_stream_dispatch.inl:69-250
// The pool is a single cudaMalloc made at init. alloc/free take one mutex
// around O(1) TLSF bookkeeping. Stream-ordered frees park the block behind a
// CUDA event until the stream passes it; parked blocks are reclaimed on the
// next alloc (at most 64 checked per call, all of them when an alloc fails).
#include "gpu/gpu_hot_runtime.h"
#include "memory/ptx_tlsf_allocator.h"

#include <cuda_runtime_api.h>

#include <cstdio>
#include <cstdlib>
#include <deque>
#include <mutex>
#include <new>
#include <vector>

struct GPUHotRuntime {
    int device = 0;
    void* pool = nullptr;
    size_t pool_size = 0;
    PTXTLSFAllocator* tlsf = nullptr;
    std::mutex mu;
    std::vector<cudaStream_t> streams;
    struct Parked { void* ptr; cudaEvent_t ev; };
    std::deque<Parked> parked;
    std::vector<cudaEvent_t> spare_events;
    bool quiet = true;
};

namespace {

size_t env_size(const char* name, size_t dflt) {
    const char* v = std::getenv(name);
    if (!v || !*v) return dflt;
    return static_cast<size_t>(std::strtoull(v, nullptr, 10));
}

// Returns parked blocks whose event has completed. Caller holds rt->mu.
void drain_parked(GPUHotRuntime* rt, int max_check) {
    int checked = 0;
    while (!rt->parked.empty() && (max_check <= 0 || checked < max_check)) {
        GPUHotRuntime::Parked& p = rt->parked.front();
        if (cudaEventQuery(p.ev) != cudaSuccess) break;  // in order per stream; stop at first pending
        ptx_tlsf_free(rt->tlsf, p.ptr);
        rt->spare_events.push_back(p.ev);
        rt->parked.pop_front();
        ++checked;
    }
}

}  // namespace

extern "C" {

GPUHotConfig gpu_hot_default_config(void) {
    GPUHotConfig c{};
    c.pool_fraction = 0.0f;
    c.fixed_pool_size = 0;
    c.min_pool_size = 256ull << 20;
    c.max_pool_size = 0;
    c.reserve_vram = 256ull << 20;
    c.enable_leak_detection = true;
    c.enable_pool_health = true;
    c.warning_threshold = 0.9f;
    c.force_daemon_mode = false;
    c.quiet_init = true;
    c.max_streams = 16;
    c.single_pool_strict = false;
    return c;
}

GPUHotRuntime* gpu_hot_init_with_config(int device_id, const char* /*token*/, const GPUHotConfig* cfg_in) {
    GPUHotConfig cfg = cfg_in ? *cfg_in : gpu_hot_default_config();
    if (cudaSetDevice(device_id) != cudaSuccess) return nullptr;
    size_t free_b = 0, total_b = 0;
    if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) return nullptr;

    size_t want = cfg.fixed_pool_size;
    if (cfg.pool_fraction > 0.0f || want == 0) {
        const float frac = cfg.pool_fraction > 0.0f ? cfg.pool_fraction : 0.7f;
        want = static_cast<size_t>(static_cast<double>(free_b) * frac);
    }
    want = env_size("PTX_POOL_SIZE", want);
    if (cfg.max_pool_size && want > cfg.max_pool_size) want = cfg.max_pool_size;
    if (want < cfg.min_pool_size && cfg.fixed_pool_size == 0) want = cfg.min_pool_size;
    const size_t reserve = cfg.reserve_vram;
    if (free_b > reserve && want > free_b - reserve) want = free_b - reserve;
    want = (want + TLSF_ALIGNMENT - 1) & ~static_cast<size_t>(TLSF_ALIGNMENT - 1);
    if (want == 0) return nullptr;

    auto* rt = new (std::nothrow) GPUHotRuntime();
    if (!rt) return nullptr;
    rt->device = device_id;
    rt->quiet = cfg.quiet_init;
    if (cudaMalloc(&rt->pool, want) != cudaSuccess) {
        cudaGetLastError();
        delete rt;
        return nullptr;
    }
    rt->pool_size = want;
    rt->tlsf = ptx_tlsf_create_from_pool(rt->pool, want, false);
    cudaStream_t s0 = nullptr;
    if (!rt->tlsf || cudaStreamCreateWithFlags(&s0, cudaStreamNonBlocking) != cudaSuccess) {
        if (rt->tlsf) ptx_tlsf_destroy(rt->tlsf);
        cudaFree(rt->pool);
        delete rt;
        return nullptr;
    }
    rt->streams.push_back(s0);
    const unsigned n = cfg.max_streams ? cfg.max_streams : 16;
    rt->streams.resize(n, nullptr);
    if (!rt->quiet)
        std::printf("[fercuda] device %d: TLSF pool %.1f MiB\n", device_id, want / 1048576.0);
    return rt;
}

GPUHotRuntime* gpu_hot_init(int device_id, const char* token) {
    return gpu_hot_init_with_config(device_id, token, nullptr);
}

void gpu_hot_shutdown(GPUHotRuntime* rt) {
    if (!rt) return;
    {
        std::lock_guard<std::mutex> lk(rt->mu);
        for (auto& p : rt->parked) {
            cudaEventSynchronize(p.ev);
            ptx_tlsf_free(rt->tlsf, p.ptr);
            cudaEventDestroy(p.ev);
        }
        rt->parked.clear();
        for (cudaEvent_t e : rt->spare_events) cudaEventDestroy(e);
        rt->spare_events.clear();
    }
    for (cudaStream_t s : rt->streams)
        if (s) { cudaStreamSynchronize(s); cudaStreamDestroy(s); }
    ptx_tlsf_destroy(rt->tlsf);
    cudaFree(rt->pool);
    delete rt;
}

void* gpu_hot_alloc(GPUHotRuntime* rt, size_t size) {
    if (!rt) return nullptr;
    std::lock_guard<std::mutex> lk(rt->mu);
    if (!rt->parked.empty()) drain_parked(rt, 64);
    void* p = ptx_tlsf_alloc(rt->tlsf, size);
    if (!p && !rt->parked.empty()) {
        drain_parked(rt, 0);
        p = ptx_tlsf_alloc(rt->tlsf, size);
    }
    return p;
}

void gpu_hot_free(GPUHotRuntime* rt, void* ptr) {
    if (!rt || !ptr) return;
    std::lock_guard<std::mutex> lk(rt->mu);
    ptx_tlsf_free(rt->tlsf, ptr);
}

void* gpu_hot_alloc_async(GPUHotRuntime* rt, size_t size, cudaStream_t) {
    // Allocation is immediate; the block is only used by work queued after
    // this call, so no stream wait is needed.
    return gpu_hot_alloc(rt, size);
}

void gpu_hot_free_async(GPUHotRuntime* rt, void* ptr, cudaStream_t stream) {
    if (!rt || !ptr) return;
    std::lock_guard<std::mutex> lk(rt->mu);
    cudaEvent_t ev = nullptr;
    if (!rt->spare_events.empty()) {
        ev = rt->spare_events.back();
        rt->spare_events.pop_back();
    } else if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) {
        // Cannot order the free: wait for the stream, then free now.
        cudaStreamSynchronize(stream);
        ptx_tlsf_free(rt->tlsf, ptr);
        return;
    }
    cudaEventRecord(ev, stream);
    rt->parked.push_back({ptr, ev});
}

void gpu_hot_poll_deferred(GPUHotRuntime* rt, int max_drain) {
    if (!rt) return;
    std::lock_guard<std::mutex> lk(rt->mu);
    drain_parked(rt, max_drain);
}

bool gpu_hot_can_allocate(GPUHotRuntime* rt, size_t size) {
    if (!rt) return false;
    std::lock_guard<std::mutex> lk(rt->mu);
    return ptx_tlsf_can_allocate(rt->tlsf, size);
}

size_t gpu_hot_get_max_allocatable(GPUHotRuntime* rt) {
    if (!rt) return 0;
    std::lock_guard<std::mutex> lk(rt->mu);
    return ptx_tlsf_get_max_allocatable(rt->tlsf);
}

bool gpu_hot_owns_ptr(GPUHotRuntime* rt, void* ptr) {
    if (!rt) return false;
    std::lock_guard<std::mutex> lk(rt->mu);
    return ptx_tlsf_owns_ptr(rt->tlsf, ptr);
}

void* gpu_hot_alloc_owned(GPUHotRuntime* rt, size_t size, uint32_t owner_id) {
    if (!rt) return nullptr;
    std::lock_guard<std::mutex> lk(rt->mu);
    return ptx_tlsf_alloc_owned(rt->tlsf, size, owner_id);
}

void gpu_hot_free_owner(GPUHotRuntime* rt, uint32_t owner_id) {
    if (!rt) return;
    std::lock_guard<std::mutex> lk(rt->mu);
    ptx_tlsf_free_owner(rt->tlsf, owner_id);
}

void gpu_hot_get_owner_stats(GPUHotRuntime* rt, TLSFOwnerStats* stats) {
    if (!rt) return;
    std::lock_guard<std::mutex> lk(rt->mu);
    ptx_tlsf_get_owner_stats(rt->tlsf, stats);
}

void gpu_hot_get_alloc_events(GPUHotRuntime* rt, TLSFEventRing* ring_out) {
    if (!rt) return;
    std::lock_guard<std::mutex> lk(rt->mu);
    ptx_tlsf_get_events(rt->tlsf, ring_out);
}

cudaStream_t gpu_hot_get_stream(GPUHotRuntime* rt, int index) {
    if (!rt || index < 0 || static_cast<size_t>(index) >= rt->streams.size()) return nullptr;
    std::lock_guard<std::mutex> lk(rt->mu);
    if (!rt->streams[index]) {
        cudaStream_t s = nullptr;
        if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) return nullptr;
        rt->streams[index] = s;
    }
    return rt->streams[index];
}

void gpu_hot_get_tlsf_stats(GPUHotRuntime* rt, TLSFPoolStats* stats) {
    if (!rt) return;
    std::lock_guard<std::mutex> lk(rt->mu);
    ptx_tlsf_get_stats(rt->tlsf, stats);
}

void gpu_hot_validate_tlsf_pool(GPUHotRuntime* rt, TLSFHealthReport* report) {
    if (!rt) return;
    std::lock_guard<std::mutex> lk(rt->mu);
    ptx_tlsf_validate(rt->tlsf, report);
}

}  // extern "C"
