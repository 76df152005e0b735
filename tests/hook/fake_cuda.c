/*
 * A stand-in for the CUDA runtime and driver allocation calls, on host
 * memory, so that libptx_hook.so's routing can be tested without a GPU.
 * Test infrastructure (tests/test_hook.py). "Device" blocks are 256-byte
 * aligned heap blocks; every block this library hands out is recorded, so a
 * free of anything else returns an error code instead of touching memory.
 * fake_cuda_calls() counts the allocations this library served.
 */
#define _GNU_SOURCE
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef int err_t;
typedef void* stream_t;
typedef unsigned long long devptr_t;

enum { kMax = 4096 };
static void* g_live[kMax];
static int g_calls;

int fake_cuda_calls(void) { return g_calls; }

static err_t take(void** p, size_t n) {
    if (!p) return 1;
    if (n == 0) {
        *p = NULL;
        return 0;
    }
    void* q = aligned_alloc(256, (n + 255) / 256 * 256);
    if (!q) return 2;
    for (int i = 0; i < kMax; ++i)
        if (!g_live[i]) {
            g_live[i] = q;
            *p = q;
            ++g_calls;
            return 0;
        }
    free(q);
    return 2;
}

static err_t give(void* p) {
    if (!p) return 0;
    for (int i = 0; i < kMax; ++i)
        if (g_live[i] == p) {
            g_live[i] = NULL;
            free(p);
            return 0;
        }
    return 1; /* not ours: invalid value */
}

err_t cudaMalloc(void** p, size_t n) { return take(p, n); }
err_t cudaFree(void* p) { return give(p); }
err_t cudaMallocAsync(void** p, size_t n, stream_t s) { (void)s; return take(p, n); }
err_t cudaFreeAsync(void* p, stream_t s) { (void)s; return give(p); }
err_t cudaMallocFromPoolAsync(void** p, size_t n, void* pool, stream_t s) { (void)pool; (void)s; return take(p, n); }
err_t cudaMallocManaged(void** p, size_t n, unsigned int f) { (void)f; return take(p, n); }
err_t cudaMallocPitch(void** p, size_t* pitch, size_t w, size_t h) {
    *pitch = (w + 511) / 512 * 512;
    return take(p, *pitch * h);
}
err_t cudaMallocHost(void** p, size_t n) { return take(p, n); }
err_t cudaHostAlloc(void** p, size_t n, unsigned int f) { (void)f; return take(p, n); }
err_t cudaFreeHost(void* p) { return give(p); }
err_t cudaMemcpy(void* d, const void* s, size_t n, int kind) { (void)kind; memcpy(d, s, n); return 0; }
err_t cudaStreamCreate(stream_t* s) { *s = (stream_t)(uintptr_t)0x51; return 0; }
err_t cudaStreamSynchronize(stream_t s) { (void)s; return 0; }
err_t cudaStreamDestroy(stream_t s) { (void)s; return 0; }
err_t cudaDeviceSynchronize(void) { return 0; }
err_t cudaSetDevice(int d) { (void)d; return 0; }
const char* cudaGetErrorString(err_t e) { (void)e; return "fake"; }

int cuMemAlloc_v2(devptr_t* p, size_t n) { void* q = NULL; int e = take(&q, n); *p = (devptr_t)(uintptr_t)q; return e; }
int cuMemFree_v2(devptr_t p) { return give((void*)(uintptr_t)p); }
int cuMemAllocAsync(devptr_t* p, size_t n, stream_t s) { (void)s; return cuMemAlloc_v2(p, n); }
int cuMemFreeAsync(devptr_t p, stream_t s) { (void)s; return cuMemFree_v2(p); }
int cuMemAllocManaged(devptr_t* p, size_t n, unsigned int f) { (void)f; return cuMemAlloc_v2(p, n); }
int cuMemAllocPitch_v2(devptr_t* p, size_t* pitch, size_t w, size_t h, unsigned int e) {
    (void)e;
    *pitch = (w + 511) / 512 * 512;
    return cuMemAlloc_v2(p, *pitch * h);
}
int cuMemAllocFromPoolAsync(devptr_t* p, size_t n, void* pool, stream_t s) { (void)pool; (void)s; return cuMemAlloc_v2(p, n); }
