/*
 * Drives libptx_hook.so through the CUDA allocation entry points and checks
 * where each allocation went. Test program: built by tests/test_hook.py
 * (against the fake CUDA and pool libraries in this folder, on the CPU) and
 * tests/test_gpu_hook.py (against the CUDA runtime and driver, on a GPU).
 *
 *   hook_driver <scenario>
 *       scenario: pool | cuda | hybrid | disabled | fallback | adopt | native
 *
 * pool      tlsf mode with a working pool: every device allocation comes from
 *           the pool, data round-trips, pitches are rounded to 256 bytes,
 *           stream-ordered and driver-API calls are served, foreign frees
 *           are refused without reaching CUDA, pinned host memory is CUDA's
 * cuda      PTX_HOOK_MODE=cuda: nothing reaches the pool
 * hybrid    PTX_HOOK_MODE=hybrid: a thread in CUDA mode bypasses the pool
 * disabled  PTX_HOOK_DISABLE=1: cudaMalloc fails, the driver API and pitched
 *           calls fall back to CUDA
 * fallback  hybrid mode with PTX_HOOK_HYBRID_FALLBACK and no pool: cudaMalloc
 *           falls back to CUDA
 * adopt     PTX_RUNTIME_PTR set (by this program, before its first
 *           allocation) to a runtime it made with gpu_hot_init: the hook
 *           serves from that runtime's pool
 * native    no hook loaded: plain CUDA behaviour of the same calls
 * Prints one line per check; exit status 0 when all pass.
 */
#define _GNU_SOURCE
#include <cuda_runtime_api.h>
#include <dlfcn.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

typedef unsigned long long devptr_t;
int cuMemAlloc_v2(devptr_t* p, size_t n);
int cuMemFree_v2(devptr_t p);
int cuMemAllocAsync(devptr_t* p, size_t n, cudaStream_t s);
int cuMemFreeAsync(devptr_t p, cudaStream_t s);
int cuMemAllocPitch_v2(devptr_t* p, size_t* pitch, size_t w, size_t h, unsigned int elem);

typedef void (*stats_fn)(uint64_t*, uint64_t*, uint64_t*);
typedef void* (*runtime_fn)(void);
typedef void (*mode_fn)(int);
typedef _Bool (*owns_fn)(void*, void*);

static int g_fail = 0;
static stats_fn hook_stats;
static runtime_fn hook_runtime;
static mode_fn hook_set_mode;
static owns_fn pool_owns;

static void check(int ok, const char* what) {
    printf("%s %s\n", ok ? "ok" : "FAIL", what);
    if (!ok) g_fail = 1;
}

static uint64_t pool_allocs(void) {
    uint64_t a = 0;
    if (hook_stats) hook_stats(&a, NULL, NULL);
    return a;
}

static uint64_t pool_frees(void) {
    uint64_t f = 0;
    if (hook_stats) hook_stats(NULL, &f, NULL);
    return f;
}

static int owned(void* p) {
    void* rt = hook_runtime ? hook_runtime() : NULL;
    return rt && pool_owns && pool_owns(rt, p);
}

static uint32_t lcg(uint32_t* s) {
    *s = *s * 1664525u + 1013904223u;
    return *s >> 8;
}

/* 48 allocations of 1 B .. 1 MiB through cudaMalloc: all succeed, are
 * 256-byte aligned and disjoint, and hold what is copied into them. Returns
 * how many the pool owns. */
static int blocks_round_trip(const char* tag) {
    enum { N = 48 };
    void* p[N];
    size_t n[N];
    uint32_t seed = 7;
    int ok = 1, own = 0;
    for (int i = 0; i < N; ++i) {
        n[i] = 1 + lcg(&seed) % (1u << 20);
        p[i] = NULL;
        ok &= cudaMalloc(&p[i], n[i]) == cudaSuccess && p[i] != NULL;
    }
    char buf[64];
    snprintf(buf, sizeof buf, "%s: cudaMalloc of 48 blocks", tag);
    check(ok, buf);
    if (!ok) return 0;
    int aligned = 1, disjoint = 1;
    for (int i = 0; i < N; ++i) {
        aligned &= ((uintptr_t)p[i] & 255u) == 0;
        own += owned(p[i]);
        for (int j = 0; j < i; ++j) {
            uintptr_t a = (uintptr_t)p[i], b = (uintptr_t)p[j];
            if (a < b + n[j] && b < a + n[i]) disjoint = 0;
        }
    }
    snprintf(buf, sizeof buf, "%s: 256-byte aligned", tag);
    check(aligned, buf);
    snprintf(buf, sizeof buf, "%s: disjoint", tag);
    check(disjoint, buf);
    int same = 1;
    for (int i = 0; i < N; ++i) {
        size_t m = n[i] < 4096 ? n[i] : 4096;
        unsigned char src[4096], dst[4096];
        for (size_t k = 0; k < m; ++k) src[k] = (unsigned char)(i * 31 + k);
        memset(dst, 0, m);
        same &= cudaMemcpy(p[i], src, m, cudaMemcpyHostToDevice) == cudaSuccess;
        same &= cudaMemcpy(dst, p[i], m, cudaMemcpyDeviceToHost) == cudaSuccess;
        same &= memcmp(src, dst, m) == 0;
    }
    snprintf(buf, sizeof buf, "%s: data round-trips", tag);
    check(same, buf);
    int freed = 1;
    for (int i = 0; i < N; ++i) freed &= cudaFree(p[i]) == cudaSuccess;
    snprintf(buf, sizeof buf, "%s: cudaFree of 48 blocks", tag);
    check(freed, buf);
    return own;
}

static void scenario_pool(void) {
    check(hook_stats && hook_runtime, "hook loaded");
    const uint64_t a0 = pool_allocs();
    check(blocks_round_trip("pool") == 48, "pool owns all 48 blocks");
    check(hook_runtime() != NULL, "pool runtime made on first allocation");
    check(pool_allocs() - a0 == 48 && pool_frees() == pool_allocs(), "stats count the pool's allocations and frees");

    void* z = (void*)1;
    check(cudaMalloc(&z, 0) == cudaSuccess && z == NULL, "0-byte cudaMalloc gives NULL");

    void* pp = NULL;
    size_t pitch = 0;
    check(cudaMallocPitch(&pp, &pitch, 1000, 7) == cudaSuccess && pitch == 1024 && owned(pp),
          "cudaMallocPitch: pitch 1024 for 1000 bytes, from the pool");
    check(cudaFree(pp) == cudaSuccess, "cudaFree of the pitched block");
    devptr_t dp = 0;
    pitch = 0;
    check(cuMemAllocPitch_v2(&dp, &pitch, 300, 3, 4) == 0 && pitch == 512 && owned((void*)(uintptr_t)dp),
          "cuMemAllocPitch: pitch 512 for 300 bytes, from the pool");
    check(cuMemFree_v2(dp) == 0, "cuMemFree of the pitched block");

    cudaStream_t s = NULL;
    check(cudaStreamCreate(&s) == cudaSuccess, "stream");
    void* ap = NULL;
    check(cudaMallocAsync(&ap, 1 << 16, s) == cudaSuccess && owned(ap), "cudaMallocAsync from the pool");
    check(cudaFreeAsync(ap, s) == cudaSuccess, "cudaFreeAsync");
    devptr_t ad = 0;
    check(cuMemAllocAsync(&ad, 1 << 16, s) == 0 && owned((void*)(uintptr_t)ad), "cuMemAllocAsync from the pool");
    check(cuMemFreeAsync(ad, s) == 0, "cuMemFreeAsync");
    check(cudaStreamSynchronize(s) == cudaSuccess && cudaStreamDestroy(s) == cudaSuccess, "stream drained");

    devptr_t d = 0;
    check(cuMemAlloc_v2(&d, 4096) == 0 && owned((void*)(uintptr_t)d), "cuMemAlloc from the pool");
    check(cuMemFree_v2(d) == 0, "cuMemFree");

    const uint64_t f0 = pool_frees();
    check(cudaFree((void*)(uintptr_t)0x1000) == cudaErrorInvalidDevicePointer, "foreign cudaFree refused");
    check(cuMemFree_v2(0x1000) == 0, "foreign cuMemFree reported, CUDA_SUCCESS");
    check(pool_frees() == f0, "foreign frees leave the pool alone");

    void* h = NULL;
    const uint64_t a1 = pool_allocs();
    check(cudaMallocHost(&h, 1 << 12) == cudaSuccess && h != NULL && !owned(h), "cudaMallocHost from CUDA");
    if (h) {
        memset(h, 0x5a, 1 << 12);
        check(cudaFreeHost(h) == cudaSuccess, "cudaFreeHost");
    }
    check(pool_allocs() == a1, "pinned host memory not counted by the pool");
}

static void scenario_cuda(void) {
    check(hook_stats != NULL, "hook loaded");
    check(blocks_round_trip("cuda mode") == 0, "no block from the pool");
    check(pool_allocs() == 0 && hook_runtime() == NULL, "pool never made");
}

static void scenario_hybrid(void) {
    check(hook_set_mode != NULL, "hook loaded");
    hook_set_mode(2);
    void* c = NULL;
    check(cudaMalloc(&c, 1 << 16) == cudaSuccess && c && !owned(c), "thread in CUDA mode: block from CUDA");
    hook_set_mode(0);
    void* t = NULL;
    check(cudaMalloc(&t, 1 << 16) == cudaSuccess && owned(t), "thread in default mode: block from the pool");
    check(cudaFree(c) == cudaSuccess && cudaFree(t) == cudaSuccess, "both freed where they came from");
    check(pool_allocs() == 1 && pool_frees() == 1, "pool counted one of each");
}

static void scenario_disabled(void) {
    void* p = (void*)1;
    check(cudaMalloc(&p, 1 << 16) == cudaErrorMemoryAllocation, "cudaMalloc fails without a pool");
    devptr_t d = 0;
    check(cuMemAlloc_v2(&d, 1 << 16) == 0 && d != 0, "cuMemAlloc falls back to CUDA");
    void* q = NULL;
    size_t pitch = 0;
    check(cudaMallocPitch(&q, &pitch, 1000, 2) == cudaSuccess && q != NULL, "cudaMallocPitch falls back to CUDA");
    check(cuMemFree_v2(d) == 0, "cuMemFree of the CUDA block");
    check(pool_allocs() == 0 && hook_runtime() == NULL, "pool never made");
    /* cudaFree of q: tlsf mode refuses a pointer the pool does not own; the
     * process exit releases it. */
}

static void scenario_fallback(void) {
    void* p = NULL;
    check(cudaMalloc(&p, 1 << 16) == cudaSuccess && p != NULL, "cudaMalloc falls back to CUDA");
    check(!owned(p) && pool_allocs() == 0, "block from CUDA");
    check(cudaFree(p) == cudaSuccess, "hybrid mode frees it through CUDA");
}

typedef void* (*init_fn)(int, const char*);

static void scenario_adopt(void) {
    init_fn init = (init_fn)dlsym(RTLD_DEFAULT, "gpu_hot_init");
    void* rt = init ? init(0, NULL) : NULL;
    check(rt != NULL, "runtime made by the program");
    if (!rt) return;
    char hex[32];
    snprintf(hex, sizeof hex, "%llx", (unsigned long long)(uintptr_t)rt);
    setenv("PTX_RUNTIME_PTR", hex, 1);
    void* p = NULL;
    check(cudaMalloc(&p, 1 << 16) == cudaSuccess && hook_runtime && hook_runtime() == rt,
          "hook adopted the program's runtime");
    check(pool_owns && pool_owns(rt, p), "block from the adopted pool");
    check(cudaFree(p) == cudaSuccess && !pool_owns(rt, p), "freed back into it");
}

static void scenario_native(void) {
    check(hook_stats == NULL, "no hook loaded");
    check(blocks_round_trip("native") == 0, "plain CUDA allocations");
}

int main(int argc, char** argv) {
    if (argc != 2) return 64;
    hook_stats = (stats_fn)dlsym(RTLD_DEFAULT, "ptx_hook_get_stats");
    hook_runtime = (runtime_fn)dlsym(RTLD_DEFAULT, "ptx_hook_get_runtime");
    hook_set_mode = (mode_fn)dlsym(RTLD_DEFAULT, "ptx_hook_set_thread_mode");
    pool_owns = (owns_fn)dlsym(RTLD_DEFAULT, "gpu_hot_owns_ptr");
    if (cudaFree(NULL) != cudaSuccess) {
        printf("FAIL context\n");
        return 2;
    }
    if (!strcmp(argv[1], "pool"))
        scenario_pool();
    else if (!strcmp(argv[1], "cuda"))
        scenario_cuda();
    else if (!strcmp(argv[1], "hybrid"))
        scenario_hybrid();
    else if (!strcmp(argv[1], "disabled"))
        scenario_disabled();
    else if (!strcmp(argv[1], "fallback"))
        scenario_fallback();
    else if (!strcmp(argv[1], "adopt"))
        scenario_adopt();
    else if (!strcmp(argv[1], "native"))
        scenario_native();
    else
        return 64;
    return g_fail;
}
