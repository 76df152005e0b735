// fer_alloc_bench: cudaMalloc + cudaFree pairs of one size, timed on the host.
//
// Run as is for CUDA's own allocator and under LD_PRELOAD=libptx_hook.so for
// the TLSF pool. The workload is that of the reference's allocator claim
// (tests/bench/bench_alloc_vs_cudamalloc.cu:21-25, 89-114): after `warmup`
// pairs, `iters` back-to-back pairs of `bytes` each, timed as one loop, and
// the same key=value lines (mode, iters, bytes, ns_per_alloc_free,
// alloc_free_per_sec, total_sec). A second pass of the same length times each
// call on its own and adds alloc / free p50 and p99 (including one
// steady_clock read, clock_ns). Under the hook, pool_allocs / pool_frees count
// the calls the pool served.
//
// Links the CUDA runtime dynamically, so that an LD_PRELOADed cudaMalloc
// takes the calls.
#include <cuda_runtime_api.h>
#include <dlfcn.h>

#include <algorithm>
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

namespace {

using Clock = std::chrono::steady_clock;

double ns_between(Clock::time_point a, Clock::time_point b) {
    return std::chrono::duration<double, std::nano>(b - a).count();
}

double pct(std::vector<double>& v, double q) {
    if (v.empty()) return 0.0;
    const size_t k = std::min(v.size() - 1, static_cast<size_t>(q * static_cast<double>(v.size())));
    std::nth_element(v.begin(), v.begin() + static_cast<long>(k), v.end());
    return v[k];
}

int fail(const char* what, int iter, cudaError_t e, int code) {
    std::fprintf(stderr, "%s failed at iteration %d: %s\n", what, iter, cudaGetErrorString(e));
    return code;
}

}  // namespace

int main(int argc, char** argv) {
    int iters = 50000, warmup = 1000;
    size_t bytes = 65536;
    for (int i = 1; i < argc; ++i) {
        if (!std::strcmp(argv[i], "--iters") && i + 1 < argc)
            iters = std::atoi(argv[++i]);
        else if (!std::strcmp(argv[i], "--bytes") && i + 1 < argc)
            bytes = static_cast<size_t>(std::strtoull(argv[++i], nullptr, 10));
        else if (!std::strcmp(argv[i], "--warmup") && i + 1 < argc)
            warmup = std::atoi(argv[++i]);
        else {
            std::printf("usage: fer_alloc_bench [--iters N] [--bytes N] [--warmup N]\n");
            return std::strcmp(argv[i], "--help") ? 64 : 0;
        }
    }
    if (iters <= 0 || warmup < 0) return 64;

    using StatsFn = void (*)(uint64_t*, uint64_t*, uint64_t*);
    auto stats = reinterpret_cast<StatsFn>(dlsym(RTLD_DEFAULT, "ptx_hook_get_stats"));

    cudaError_t e = cudaSetDevice(0);
    if (e != cudaSuccess) return fail("cudaSetDevice", -1, e, 1);
    e = cudaFree(nullptr);
    if (e != cudaSuccess) return fail("cudaFree(NULL)", -1, e, 2);

    for (int i = 0; i < warmup; ++i) {
        void* p = nullptr;
        if ((e = cudaMalloc(&p, bytes)) != cudaSuccess) return fail("warm-up cudaMalloc", i, e, 3);
        if ((e = cudaFree(p)) != cudaSuccess) return fail("warm-up cudaFree", i, e, 4);
    }

    const Clock::time_point t0 = Clock::now();
    for (int i = 0; i < iters; ++i) {
        void* p = nullptr;
        if ((e = cudaMalloc(&p, bytes)) != cudaSuccess) return fail("cudaMalloc", i, e, 5);
        if ((e = cudaFree(p)) != cudaSuccess) return fail("cudaFree", i, e, 6);
    }
    const Clock::time_point t1 = Clock::now();
    const double total_ns = ns_between(t0, t1);

    std::vector<double> a_ns(static_cast<size_t>(iters)), f_ns(static_cast<size_t>(iters));
    for (int i = 0; i < iters; ++i) {
        void* p = nullptr;
        const Clock::time_point c0 = Clock::now();
        e = cudaMalloc(&p, bytes);
        const Clock::time_point c1 = Clock::now();
        if (e != cudaSuccess) return fail("cudaMalloc (per-call pass)", i, e, 7);
        e = cudaFree(p);
        const Clock::time_point c2 = Clock::now();
        if (e != cudaSuccess) return fail("cudaFree (per-call pass)", i, e, 8);
        a_ns[static_cast<size_t>(i)] = ns_between(c0, c1);
        f_ns[static_cast<size_t>(i)] = ns_between(c1, c2);
    }
    // Cost of one clock read, the floor under each per-call sample.
    double clock_ns = 0.0;
    {
        const int n = 100000;
        Clock::time_point c = Clock::now();
        const Clock::time_point s0 = c;
        for (int i = 0; i < n; ++i) c = std::max(c, Clock::now());
        clock_ns = ns_between(s0, c) / n;
    }

    const double per = total_ns / iters;
    std::printf("mode=%s\n", stats ? "tlsf" : "cudaMalloc");
    std::printf("iters=%d\n", iters);
    std::printf("bytes=%zu\n", bytes);
    std::printf("ns_per_alloc_free=%.1f\n", per);
    std::printf("alloc_free_per_sec=%.0f\n", 1e9 / per);
    std::printf("total_sec=%.4f\n", total_ns / 1e9);
    std::printf("alloc_p50_ns=%.1f\n", pct(a_ns, 0.50));
    std::printf("alloc_p99_ns=%.1f\n", pct(a_ns, 0.99));
    std::printf("free_p50_ns=%.1f\n", pct(f_ns, 0.50));
    std::printf("free_p99_ns=%.1f\n", pct(f_ns, 0.99));
    std::printf("clock_ns=%.1f\n", clock_ns);
    if (stats) {
        uint64_t na = 0, nf = 0, nb = 0;
        stats(&na, &nf, &nb);
        std::printf("pool_allocs=%llu\n", static_cast<unsigned long long>(na));
        std::printf("pool_frees=%llu\n", static_cast<unsigned long long>(nf));
    }
    return 0;
}
