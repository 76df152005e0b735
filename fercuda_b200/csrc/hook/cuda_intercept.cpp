// libptx_hook.so: an LD_PRELOAD interposer that serves a process's device
// allocations from the TLSF pool of libptx_core.so (gpu_hot_*).
//
//   LD_PRELOAD=libptx_hook.so ./app        (or python train.py)
//
// Replaces native/core/hooks/cuda_intercept.c:
//   environment and modes          :11-16, :326-356
//   lazy runtime creation          :239-324 (PTX_RUNTIME_PTR reuse :271-280)
//   runtime-API entry points       :377-634, :784-940
//   driver-API entry points        :636-782, :942-1066
// Kept from the reference, entry point by entry point: which calls the pool
// serves; which of them fall back to CUDA when the pool cannot be made (the
// driver API, pitched and pool-ordered calls) and which then fail (cudaMalloc,
// cudaMallocAsync, unless hybrid mode with PTX_HOOK_HYBRID_FALLBACK); pitches
// rounded up to 256 bytes; managed and pinned-host memory always from CUDA;
// a pointer the pool does not own goes to CUDA in cuda and hybrid mode, and in
// tlsf mode is reported on stderr and refused (cudaErrorInvalidDevicePointer
// from the runtime API, CUDA_SUCCESS from the driver API, as there).
// Different on purpose:
//   - cudaFree(NULL) goes to CUDA, which is how programs create the context;
//   - a 0-byte allocation returns NULL and success, as CUDA does;
//   - cuMemAllocAsync / cuMemFreeAsync are stream-ordered like the runtime
//     pair (the reference serves them synchronously);
//   - calls made while the pool's own runtime is inside CUDA go to CUDA;
//   - nothing is printed unless PTX_HOOK_VERBOSE is set;
//   - the pool is not torn down when the library unloads, so frees issued by
//     other destructors at exit still find it; process exit releases it.
// A free returns the block to the pool at once, as in the reference: work
// still queued on a non-blocking stream must not touch a block after its
// cudaFree (use cudaFreeAsync on that stream).
#ifndef _GNU_SOURCE
#define _GNU_SOURCE
#endif
#include "gpu/gpu_hot_runtime.h"
#include "ptx_hook.h"

#include <cuda_runtime_api.h>
#include <dlfcn.h>
#include <strings.h>

#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <mutex>

namespace {

// Driver-API types, declared here rather than taken from cuda.h, whose
// macros rename cuMemAlloc and friends to their _v2 forms.
using CUresult = int;
using CUdeviceptr = unsigned long long;
using CUstream = cudaStream_t;
using CUmemoryPool = cudaMemPool_t;
constexpr CUresult kCuSuccess = 0;
constexpr CUresult kCuOutOfMemory = 2;

enum Mode { kModeTlsf = 0, kModeCuda = 1, kModeHybrid = 2 };
enum State { kDisabled = -1, kUninit = 0, kReady = 2 };

Mode g_mode = kModeTlsf;
bool g_fallback = false;
bool g_verbose = false;
std::atomic<int> g_state{kUninit};
GPUHotRuntime* g_rt = nullptr;
std::mutex g_init_mu;
std::atomic<uint64_t> g_allocs{0}, g_frees{0}, g_bytes{0};
thread_local int t_guard = 0;  // > 0 while the pool runtime runs on this thread
thread_local int t_mode = PTX_HOOK_THREAD_DEFAULT;

struct Guard {
    Guard() { ++t_guard; }
    ~Guard() { --t_guard; }
};

bool env_set(const char* name) { return std::getenv(name) != nullptr; }

// ---------------------------------------------------------------- real CUDA
enum Fn {
    kMalloc, kFree, kMallocAsync, kFreeAsync, kMallocFromPoolAsync, kMallocManaged, kMallocPitch,
    kMallocHost, kHostAlloc, kFreeHost,
    kCuMemAlloc, kCuMemFree, kCuMemAllocAsync, kCuMemFreeAsync, kCuMemAllocManaged, kCuMemAllocPitch,
    kCuMemAllocFromPoolAsync, kFnCount
};

struct FnName {
    const char* name;
    const char* alt;  // tried only when `name` is missing
    bool driver;
};

// The driver's unversioned cuMemAlloc / cuMemFree / cuMemAllocPitch may call
// the _v2 symbols, which would come back here: the _v2 names come first.
constexpr FnName kNames[kFnCount] = {
    {"cudaMalloc", nullptr, false},
    {"cudaFree", nullptr, false},
    {"cudaMallocAsync", nullptr, false},
    {"cudaFreeAsync", nullptr, false},
    {"cudaMallocFromPoolAsync", nullptr, false},
    {"cudaMallocManaged", nullptr, false},
    {"cudaMallocPitch", nullptr, false},
    {"cudaMallocHost", nullptr, false},
    {"cudaHostAlloc", nullptr, false},
    {"cudaFreeHost", nullptr, false},
    {"cuMemAlloc_v2", "cuMemAlloc", true},
    {"cuMemFree_v2", "cuMemFree", true},
    {"cuMemAllocAsync", nullptr, true},
    {"cuMemFreeAsync", nullptr, true},
    {"cuMemAllocManaged", nullptr, true},
    {"cuMemAllocPitch_v2", "cuMemAllocPitch", true},
    {"cuMemAllocFromPoolAsync", nullptr, true},
};

std::atomic<void*> g_real[kFnCount];

bool is_self(void* p) {
    Dl_info a{}, b{};
    return dladdr(p, &a) && dladdr(reinterpret_cast<void*>(&is_self), &b) && a.dli_fbase == b.dli_fbase;
}

void* lookup(const char* name, bool driver) {
    if (void* p = dlsym(RTLD_NEXT, name)) return p;
    // A runtime loaded with RTLD_LOCAL (by dlopen) is not on the RTLD_NEXT
    // path; ask it by handle if it is loaded.
    static const char* const kRuntime[] = {"libcudart.so.12", "libcudart.so"};
    static const char* const kDriver[] = {"libcuda.so.1", "libcuda.so"};
    const char* const* libs = driver ? kDriver : kRuntime;
    for (int i = 0; i < 2; ++i) {
        void* h = dlopen(libs[i], RTLD_NOW | RTLD_NOLOAD);
        if (!h) continue;
        void* p = dlsym(h, name);
        dlclose(h);
        if (p) return p;
    }
    return nullptr;
}

template <class F>
F real(Fn f) {
    void* p = g_real[f].load(std::memory_order_acquire);
    if (!p) {
        p = lookup(kNames[f].name, kNames[f].driver);
        if (!p && kNames[f].alt) p = lookup(kNames[f].alt, kNames[f].driver);
        if (p && is_self(p)) p = nullptr;
        if (p) g_real[f].store(p, std::memory_order_release);
    }
    return reinterpret_cast<F>(p);
}

using MallocFn = cudaError_t (*)(void**, size_t);
using FreeFn = cudaError_t (*)(void*);
using MallocAsyncFn = cudaError_t (*)(void**, size_t, cudaStream_t);
using FreeAsyncFn = cudaError_t (*)(void*, cudaStream_t);
using MallocFromPoolFn = cudaError_t (*)(void**, size_t, cudaMemPool_t, cudaStream_t);
using MallocManagedFn = cudaError_t (*)(void**, size_t, unsigned int);
using MallocPitchFn = cudaError_t (*)(void**, size_t*, size_t, size_t);
using HostAllocFn = cudaError_t (*)(void**, size_t, unsigned int);
using CuAllocFn = CUresult (*)(CUdeviceptr*, size_t);
using CuFreeFn = CUresult (*)(CUdeviceptr);
using CuAllocAsyncFn = CUresult (*)(CUdeviceptr*, size_t, CUstream);
using CuFreeAsyncFn = CUresult (*)(CUdeviceptr, CUstream);
using CuAllocManagedFn = CUresult (*)(CUdeviceptr*, size_t, unsigned int);
using CuAllocPitchFn = CUresult (*)(CUdeviceptr*, size_t*, size_t, size_t, unsigned int);
using CuAllocFromPoolFn = CUresult (*)(CUdeviceptr*, size_t, CUmemoryPool, CUstream);

// ---------------------------------------------------------------- the pool
bool to_cuda() {
    return g_mode == kModeCuda || (g_mode == kModeHybrid && t_mode == PTX_HOOK_THREAD_CUDA);
}
bool fallback_ok() { return g_mode == kModeHybrid && g_fallback; }

// Makes (or adopts) the pool runtime on first use. False: there is no pool
// (PTX_HOOK_DISABLE, or the runtime could not be made; both are final).
bool ensure_pool() {
    const int s = g_state.load(std::memory_order_acquire);
    if (s == kReady) return true;
    if (s == kDisabled) return false;
    std::lock_guard<std::mutex> lk(g_init_mu);
    if (g_state.load(std::memory_order_relaxed) != kUninit) return g_state.load() == kReady;
    if (env_set("PTX_HOOK_DISABLE")) {
        if (g_verbose) std::fprintf(stderr, "[ptx_hook] disabled by PTX_HOOK_DISABLE\n");
        g_state.store(kDisabled, std::memory_order_release);
        return false;
    }
    GPUHotRuntime* rt = nullptr;
    const char* adopt = std::getenv("PTX_RUNTIME_PTR");
    if (adopt && *adopt) {
        rt = reinterpret_cast<GPUHotRuntime*>(static_cast<uintptr_t>(std::strtoull(adopt, nullptr, 16)));
    } else {
        const char* dev = std::getenv("PTX_HOOK_DEVICE");
        Guard g;  // the runtime's own CUDA allocations (the pool itself) go to CUDA
        rt = gpu_hot_init(dev ? std::atoi(dev) : 0, nullptr);
    }
    if (!rt) {
        std::fprintf(stderr, "[ptx_hook] could not make the TLSF pool runtime\n");
        g_state.store(kDisabled, std::memory_order_release);
        return false;
    }
    g_rt = rt;
    g_state.store(kReady, std::memory_order_release);
    if (g_verbose)
        std::fprintf(stderr, "[ptx_hook] pool runtime %p ready (%s)\n", static_cast<void*>(rt),
                     g_mode == kModeHybrid ? "hybrid" : "tlsf");
    return true;
}

enum class Route { kPool, kCuda, kFail };

// Where an allocation goes before the pool is tried. init_fail_to_cuda: the
// entry point uses CUDA when the pool cannot be made.
Route route(bool init_fail_to_cuda) {
    if (t_guard || to_cuda()) return Route::kCuda;
    if (ensure_pool()) return Route::kPool;
    return init_fail_to_cuda || fallback_ok() ? Route::kCuda : Route::kFail;
}

void* pool_alloc(size_t bytes, cudaStream_t stream, bool ordered) {
    Guard g;
    void* p = ordered ? gpu_hot_alloc_async(g_rt, bytes, stream) : gpu_hot_alloc(g_rt, bytes);
    if (p) {
        g_allocs.fetch_add(1, std::memory_order_relaxed);
        g_bytes.fetch_add(bytes, std::memory_order_relaxed);
    }
    return p;
}

// True when the pool owns p and has taken it back.
bool pool_free(void* p, cudaStream_t stream, bool ordered) {
    if (t_guard || g_state.load(std::memory_order_acquire) != kReady) return false;
    Guard g;
    if (!gpu_hot_owns_ptr(g_rt, p)) return false;
    if (ordered)
        gpu_hot_free_async(g_rt, p, stream);
    else
        gpu_hot_free(g_rt, p);
    g_frees.fetch_add(1, std::memory_order_relaxed);
    return true;
}

void report_foreign_free(const char* fn, const void* p) {
    std::fprintf(stderr, "[ptx_hook] %s: %p is not a pool pointer (tlsf mode); refused\n", fn, p);
}

// One allocation entry point: the pool when routed there (`set` stores the
// pointer), else `cuda()`; `fail` when neither may serve it.
template <class R, class Set, class Cuda>
R serve(const char* fn, size_t bytes, cudaStream_t stream, bool ordered, bool init_fail_to_cuda, R fail, Set set,
        Cuda cuda) {
    switch (route(init_fail_to_cuda)) {
        case Route::kCuda: return cuda();
        case Route::kFail: return fail;
        case Route::kPool: break;
    }
    if (bytes == 0) {
        set(nullptr);
        return R(0);
    }
    if (void* p = pool_alloc(bytes, stream, ordered)) {
        set(p);
        if (g_verbose) std::fprintf(stderr, "[ptx_hook] %s(%zu) = %p\n", fn, bytes, p);
        return R(0);
    }
    if (g_verbose) std::fprintf(stderr, "[ptx_hook] %s(%zu): pool has no room\n", fn, bytes);
    return fallback_ok() ? cuda() : fail;
}

auto set_ptr(void** out) {
    return [out](void* p) { *out = p; };
}
auto set_dptr(CUdeviceptr* out) {
    return [out](void* p) { *out = static_cast<CUdeviceptr>(reinterpret_cast<uintptr_t>(p)); };
}

bool pitch_bytes(size_t width, size_t height, size_t* pitch, size_t* total) {
    if (width > SIZE_MAX - 255) return false;
    *pitch = (width + 255) / 256 * 256;
    if (height && *pitch > SIZE_MAX / height) return false;
    *total = *pitch * height;
    return true;
}

__attribute__((constructor)) void hook_load() {
    g_verbose = env_set("PTX_HOOK_VERBOSE");
    if (const char* m = std::getenv("PTX_HOOK_MODE")) {
        if (strcasecmp(m, "cuda") == 0)
            g_mode = kModeCuda;
        else if (strcasecmp(m, "hybrid") == 0)
            g_mode = kModeHybrid;
    }
    g_fallback = env_set("PTX_HOOK_HYBRID_FALLBACK");
    if (g_verbose)
        std::fprintf(stderr, "[ptx_hook] loaded, mode %s\n",
                     g_mode == kModeCuda ? "cuda" : g_mode == kModeHybrid ? "hybrid" : "tlsf");
}

__attribute__((destructor)) void hook_unload() {
    if (g_verbose)
        std::fprintf(stderr, "[ptx_hook] pool allocations %llu, frees %llu, bytes %llu\n",
                     static_cast<unsigned long long>(g_allocs.load()), static_cast<unsigned long long>(g_frees.load()),
                     static_cast<unsigned long long>(g_bytes.load()));
}

}  // namespace

extern "C" {

// ---------------------------------------------------------------- control API
void ptx_hook_set_thread_mode(int mode) { t_mode = mode; }
int ptx_hook_get_thread_mode(void) { return t_mode; }

void ptx_hook_get_stats(uint64_t* allocs, uint64_t* frees, uint64_t* bytes) {
    if (allocs) *allocs = g_allocs.load(std::memory_order_relaxed);
    if (frees) *frees = g_frees.load(std::memory_order_relaxed);
    if (bytes) *bytes = g_bytes.load(std::memory_order_relaxed);
}

void* ptx_hook_get_runtime(void) {
    return g_state.load(std::memory_order_acquire) == kReady ? static_cast<void*>(g_rt) : nullptr;
}

// ---------------------------------------------------------------- runtime API
cudaError_t cudaMalloc(void** devPtr, size_t size) {
    if (!devPtr) return cudaSuccess;
    return serve("cudaMalloc", size, nullptr, false, false, cudaErrorMemoryAllocation, set_ptr(devPtr), [&] {
        auto f = real<MallocFn>(kMalloc);
        return f ? f(devPtr, size) : cudaErrorMemoryAllocation;
    });
}

cudaError_t cudaFree(void* devPtr) {
    auto cuda = [&] {
        auto f = real<FreeFn>(kFree);
        return f ? f(devPtr) : (devPtr ? cudaErrorInvalidDevicePointer : cudaSuccess);
    };
    if (!devPtr || t_guard) return cuda();
    if (pool_free(devPtr, nullptr, false)) return cudaSuccess;
    if (to_cuda() || g_mode == kModeHybrid) return cuda();
    report_foreign_free("cudaFree", devPtr);
    return cudaErrorInvalidDevicePointer;
}

cudaError_t cudaMallocAsync(void** devPtr, size_t size, cudaStream_t stream) {
    if (!devPtr) return cudaSuccess;
    return serve("cudaMallocAsync", size, stream, true, false, cudaErrorMemoryAllocation, set_ptr(devPtr), [&] {
        if (auto f = real<MallocAsyncFn>(kMallocAsync)) return f(devPtr, size, stream);
        auto g = real<MallocFn>(kMalloc);
        return g ? g(devPtr, size) : cudaErrorMemoryAllocation;
    });
}

cudaError_t cudaFreeAsync(void* devPtr, cudaStream_t stream) {
    if (!devPtr) return cudaSuccess;
    auto cuda = [&] {
        if (auto f = real<FreeAsyncFn>(kFreeAsync)) return f(devPtr, stream);
        auto g = real<FreeFn>(kFree);
        return g ? g(devPtr) : cudaErrorInvalidDevicePointer;
    };
    if (t_guard) return cuda();
    if (pool_free(devPtr, stream, true)) return cudaSuccess;
    if (to_cuda() || g_mode == kModeHybrid) return cuda();
    report_foreign_free("cudaFreeAsync", devPtr);
    return cudaErrorInvalidDevicePointer;
}

cudaError_t cudaMallocFromPoolAsync(void** devPtr, size_t size, cudaMemPool_t memPool, cudaStream_t stream) {
    if (!devPtr) return cudaSuccess;
    // The CUDA pool is ignored: its memory would not be TLSF memory.
    return serve("cudaMallocFromPoolAsync", size, stream, true, true, cudaErrorMemoryAllocation, set_ptr(devPtr),
                 [&] {
        auto f = real<MallocFromPoolFn>(kMallocFromPoolAsync);
        return f ? f(devPtr, size, memPool, stream) : cudaErrorMemoryAllocation;
    });
}

cudaError_t cudaMallocPitch(void** devPtr, size_t* pitch, size_t width, size_t height) {
    if (!devPtr || !pitch) return cudaSuccess;
    auto cuda = [&] {
        auto f = real<MallocPitchFn>(kMallocPitch);
        return f ? f(devPtr, pitch, width, height) : cudaErrorMemoryAllocation;
    };
    const Route r = route(true);
    if (r == Route::kCuda) return cuda();
    size_t p = 0, total = 0;
    if (r == Route::kFail || !pitch_bytes(width, height, &p, &total)) return cudaErrorMemoryAllocation;
    if (total == 0) {
        *devPtr = nullptr;
        *pitch = p;
        return cudaSuccess;
    }
    if (void* ptr = pool_alloc(total, nullptr, false)) {
        *devPtr = ptr;
        *pitch = p;
        return cudaSuccess;
    }
    return fallback_ok() ? cuda() : cudaErrorMemoryAllocation;
}

cudaError_t cudaMallocManaged(void** devPtr, size_t size, unsigned int flags) {
    auto f = real<MallocManagedFn>(kMallocManaged);
    return f ? f(devPtr, size, flags) : cudaErrorMemoryAllocation;
}

cudaError_t cudaMallocHost(void** ptr, size_t size) {
    auto f = real<MallocFn>(kMallocHost);
    return f ? f(ptr, size) : cudaErrorMemoryAllocation;
}

cudaError_t cudaHostAlloc(void** pHost, size_t size, unsigned int flags) {
    auto f = real<HostAllocFn>(kHostAlloc);
    return f ? f(pHost, size, flags) : cudaErrorMemoryAllocation;
}

cudaError_t cudaFreeHost(void* ptr) {
    auto f = real<FreeFn>(kFreeHost);
    return f ? f(ptr) : cudaSuccess;
}

// ---------------------------------------------------------------- driver API
CUresult cuMemAlloc_v2(CUdeviceptr* dptr, size_t bytesize) {
    if (!dptr) return kCuSuccess;
    return serve("cuMemAlloc", bytesize, nullptr, false, true, kCuOutOfMemory, set_dptr(dptr), [&] {
        auto f = real<CuAllocFn>(kCuMemAlloc);
        return f ? f(dptr, bytesize) : kCuOutOfMemory;
    });
}

CUresult cuMemAlloc(CUdeviceptr* dptr, size_t bytesize) { return cuMemAlloc_v2(dptr, bytesize); }

CUresult cuMemFree_v2(CUdeviceptr dptr) {
    void* p = reinterpret_cast<void*>(static_cast<uintptr_t>(dptr));
    auto cuda = [&] {
        auto f = real<CuFreeFn>(kCuMemFree);
        return f ? f(dptr) : kCuSuccess;
    };
    if (!p) return kCuSuccess;
    if (t_guard) return cuda();
    if (pool_free(p, nullptr, false)) return kCuSuccess;
    if (to_cuda() || g_mode == kModeHybrid) return cuda();
    report_foreign_free("cuMemFree", p);
    return kCuSuccess;
}

CUresult cuMemFree(CUdeviceptr dptr) { return cuMemFree_v2(dptr); }

CUresult cuMemAllocAsync(CUdeviceptr* dptr, size_t bytesize, CUstream hStream) {
    if (!dptr) return kCuSuccess;
    return serve("cuMemAllocAsync", bytesize, hStream, true, true, kCuOutOfMemory, set_dptr(dptr), [&] {
                     if (auto f = real<CuAllocAsyncFn>(kCuMemAllocAsync)) return f(dptr, bytesize, hStream);
                     auto g = real<CuAllocFn>(kCuMemAlloc);
                     return g ? g(dptr, bytesize) : kCuOutOfMemory;
                 });
}

CUresult cuMemFreeAsync(CUdeviceptr dptr, CUstream hStream) {
    void* p = reinterpret_cast<void*>(static_cast<uintptr_t>(dptr));
    auto cuda = [&] {
        if (auto f = real<CuFreeAsyncFn>(kCuMemFreeAsync)) return f(dptr, hStream);
        auto g = real<CuFreeFn>(kCuMemFree);
        return g ? g(dptr) : kCuSuccess;
    };
    if (!p) return kCuSuccess;
    if (t_guard) return cuda();
    if (pool_free(p, hStream, true)) return kCuSuccess;
    if (to_cuda() || g_mode == kModeHybrid) return cuda();
    report_foreign_free("cuMemFreeAsync", p);
    return kCuSuccess;
}

CUresult cuMemAllocManaged(CUdeviceptr* dptr, size_t bytesize, unsigned int flags) {
    auto f = real<CuAllocManagedFn>(kCuMemAllocManaged);
    return f ? f(dptr, bytesize, flags) : kCuOutOfMemory;
}

CUresult cuMemAllocPitch_v2(CUdeviceptr* dptr, size_t* pPitch, size_t WidthInBytes, size_t Height,
                            unsigned int ElementSizeBytes) {
    if (!dptr || !pPitch) return kCuSuccess;
    auto cuda = [&] {
        auto f = real<CuAllocPitchFn>(kCuMemAllocPitch);
        return f ? f(dptr, pPitch, WidthInBytes, Height, ElementSizeBytes) : kCuOutOfMemory;
    };
    const Route r = route(true);
    if (r == Route::kCuda) return cuda();
    size_t p = 0, total = 0;
    if (r == Route::kFail || !pitch_bytes(WidthInBytes, Height, &p, &total)) return kCuOutOfMemory;
    if (total == 0) {
        *dptr = 0;
        *pPitch = p;
        return kCuSuccess;
    }
    if (void* ptr = pool_alloc(total, nullptr, false)) {
        *dptr = static_cast<CUdeviceptr>(reinterpret_cast<uintptr_t>(ptr));
        *pPitch = p;
        return kCuSuccess;
    }
    return fallback_ok() ? cuda() : kCuOutOfMemory;
}

CUresult cuMemAllocPitch(CUdeviceptr* dptr, size_t* pPitch, size_t WidthInBytes, size_t Height,
                         unsigned int ElementSizeBytes) {
    return cuMemAllocPitch_v2(dptr, pPitch, WidthInBytes, Height, ElementSizeBytes);
}

CUresult cuMemAllocFromPoolAsync(CUdeviceptr* dptr, size_t bytesize, CUmemoryPool pool, CUstream hStream) {
    if (!dptr) return kCuSuccess;
    return serve("cuMemAllocFromPoolAsync", bytesize, hStream, true, true, kCuOutOfMemory, set_dptr(dptr), [&] {
                     auto f = real<CuAllocFromPoolFn>(kCuMemAllocFromPoolAsync);
                     return f ? f(dptr, bytesize, pool, hStream) : kCuOutOfMemory;
                 });
}

}  // extern "C"
