// Allocation-trace replay for the pool benchmark (config: 1M alloc/free ops,
// log-uniform 256 B - 16 MiB, each allocation touched by a fill kernel).
//
// The reference measures its pool the same way in
// tests/bench/bench_alloc_vs_cudamalloc.cu:21-25,89-114 (alloc + free pairs
// timed on the host, TLSF against cudaMalloc / cudaFree). Here one routine
// replays an allocator-independent trace (positive entry = allocate that many
// bytes, negative entry = free the (-e-1)-th allocation) through either
//   - a gpu_hot runtime (the TLSF pool every fercuda buffer comes from), or
//   - cudaMalloc / cudaFree,
// launching fer_fill_u32 over each fresh block on `stream`, and records the
// host latency of every alloc and every free call in nanoseconds.
#include "gpu/gpu_hot_runtime.h"

#include <cuda_runtime_api.h>

#include <cstdint>
#include <ctime>
#include <vector>

extern "C" cudaError_t fer_fill_u32(void* dst, size_t bytes, uint32_t value, cudaStream_t stream);

namespace {

inline uint64_t now_ns() {
    timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return static_cast<uint64_t>(ts.tv_sec) * 1000000000ull + static_cast<uint64_t>(ts.tv_nsec);
}

}  // namespace

// Returns 0 on success, 1 if an allocation failed (stops there), 2 on a CUDA
// error. alloc_ns / free_ns must hold one slot per alloc / free op of the
// trace; *n_alloc / *n_free receive how many were written.
extern "C" int fer_bench_pool_replay(GPUHotRuntime* rt, int use_cuda_malloc, const int64_t* trace, size_t n,
                                     int fill_each, cudaStream_t stream, uint32_t* alloc_ns, size_t* n_alloc,
                                     uint32_t* free_ns, size_t* n_free, uint64_t* fill_bytes, double* wall_s) {
    std::vector<void*> ptrs;
    ptrs.reserve(n);
    size_t na = 0, nf = 0;
    uint64_t filled = 0;
    int rc = 0;
    const uint64_t t_start = now_ns();
    for (size_t i = 0; i < n; ++i) {
        const int64_t e = trace[i];
        if (e > 0) {
            const size_t bytes = static_cast<size_t>(e);
            void* p = nullptr;
            const uint64_t t0 = now_ns();
            if (use_cuda_malloc) {
                if (cudaMalloc(&p, bytes) != cudaSuccess) p = nullptr;
            } else {
                p = gpu_hot_alloc(rt, bytes);
            }
            const uint64_t t1 = now_ns();
            alloc_ns[na++] = static_cast<uint32_t>(t1 - t0 > 0xFFFFFFFFull ? 0xFFFFFFFFull : t1 - t0);
            ptrs.push_back(p);
            if (!p) {
                cudaGetLastError();
                rc = 1;
                break;
            }
            if (fill_each) {
                if (fer_fill_u32(p, bytes, static_cast<uint32_t>(i), stream) != cudaSuccess) {
                    rc = 2;
                    break;
                }
                filled += bytes;
            }
        } else {
            void* p = ptrs[static_cast<size_t>(-e - 1)];
            const uint64_t t0 = now_ns();
            if (use_cuda_malloc) cudaFree(p);
            else gpu_hot_free(rt, p);
            const uint64_t t1 = now_ns();
            free_ns[nf++] = static_cast<uint32_t>(t1 - t0 > 0xFFFFFFFFull ? 0xFFFFFFFFull : t1 - t0);
            ptrs[static_cast<size_t>(-e - 1)] = nullptr;
        }
    }
    if (cudaStreamSynchronize(stream) != cudaSuccess && rc == 0) rc = 2;
    *wall_s = static_cast<double>(now_ns() - t_start) * 1e-9;
    // release what is still live
    for (void* p : ptrs)
        if (p) {
            if (use_cuda_malloc) cudaFree(p);
            else gpu_hot_free(rt, p);
        }
    *n_alloc = na;
    *n_free = nf;
    *fill_bytes = filled;
    return rc;
}

// Host-only replay of the same trace through any allocator exposed as a pair
// of C function pointers (e.g. ptx_tlsf_alloc / ptx_tlsf_free of a pool
// created over a fake address range): per-op latency of the allocator's
// bookkeeping alone, without a Python call in the timed region.
using fer_bench_alloc_fn = void* (*)(void* ctx, size_t bytes);
using fer_bench_free_fn = void (*)(void* ctx, void* p);

extern "C" int fer_bench_fn_replay(fer_bench_alloc_fn alloc_fn, fer_bench_free_fn free_fn, void* ctx,
                                   const int64_t* trace, size_t n, uint32_t* alloc_ns, size_t* n_alloc,
                                   uint32_t* free_ns, size_t* n_free, double* wall_s) {
    std::vector<void*> ptrs;
    ptrs.reserve(n);
    size_t na = 0, nf = 0;
    int rc = 0;
    const uint64_t t_start = now_ns();
    for (size_t i = 0; i < n; ++i) {
        const int64_t e = trace[i];
        if (e > 0) {
            const uint64_t t0 = now_ns();
            void* p = alloc_fn(ctx, static_cast<size_t>(e));
            const uint64_t t1 = now_ns();
            alloc_ns[na++] = static_cast<uint32_t>(t1 - t0 > 0xFFFFFFFFull ? 0xFFFFFFFFull : t1 - t0);
            ptrs.push_back(p);
            if (!p) {
                rc = 1;
                break;
            }
        } else {
            void* p = ptrs[static_cast<size_t>(-e - 1)];
            const uint64_t t0 = now_ns();
            free_fn(ctx, p);
            const uint64_t t1 = now_ns();
            free_ns[nf++] = static_cast<uint32_t>(t1 - t0 > 0xFFFFFFFFull ? 0xFFFFFFFFull : t1 - t0);
            ptrs[static_cast<size_t>(-e - 1)] = nullptr;
        }
    }
    *wall_s = static_cast<double>(now_ns() - t_start) * 1e-9;
    for (void* p : ptrs)
        if (p) free_fn(ctx, p);
    *n_alloc = na;
    *n_free = nf;
    return rc;
}
