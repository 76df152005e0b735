/*
 * gpu_hot_* over a host-memory range, for testing libptx_hook.so without a
 * GPU. Test infrastructure (tests/test_hook.py): preloaded after the hook,
 * it takes the hook's gpu_hot_* calls, and carves its range with
 * libptx_core.so's own TLSF allocator (ptx_tlsf_*), which keeps its
 * bookkeeping on the host. Streams are ignored (frees are immediate).
 * FAKE_HOT_FAIL=1 makes gpu_hot_init fail.
 */
#include <stdbool.h>
#include <stdint.h>
#include <stdlib.h>

typedef struct PTXTLSFAllocator PTXTLSFAllocator;
PTXTLSFAllocator* ptx_tlsf_create_from_pool(void* pool, size_t size, bool debug_mode);
void* ptx_tlsf_alloc(PTXTLSFAllocator* a, size_t size);
void ptx_tlsf_free(PTXTLSFAllocator* a, void* p);
bool ptx_tlsf_owns_ptr(PTXTLSFAllocator* a, void* p);

typedef struct GPUHotRuntime {
    PTXTLSFAllocator* tlsf;
    void* base;
} GPUHotRuntime;

GPUHotRuntime* gpu_hot_init(int device, const char* token) {
    (void)device;
    (void)token;
    if (getenv("FAKE_HOT_FAIL")) return NULL;
    const size_t size = 64u << 20;
    GPUHotRuntime* rt = calloc(1, sizeof *rt);
    rt->base = aligned_alloc(4096, size);
    rt->tlsf = ptx_tlsf_create_from_pool(rt->base, size, false);
    return rt->tlsf ? rt : NULL;
}
void* gpu_hot_alloc(GPUHotRuntime* rt, size_t n) { return ptx_tlsf_alloc(rt->tlsf, n); }
void* gpu_hot_alloc_async(GPUHotRuntime* rt, size_t n, void* s) { (void)s; return ptx_tlsf_alloc(rt->tlsf, n); }
void gpu_hot_free(GPUHotRuntime* rt, void* p) { ptx_tlsf_free(rt->tlsf, p); }
void gpu_hot_free_async(GPUHotRuntime* rt, void* p, void* s) { (void)s; ptx_tlsf_free(rt->tlsf, p); }
bool gpu_hot_owns_ptr(GPUHotRuntime* rt, void* p) { return rt && ptx_tlsf_owns_ptr(rt->tlsf, p); }
