/*
 * Control API of libptx_hook.so, the LD_PRELOAD interposer that serves a
 * process's device allocations (cudaMalloc, cudaMallocAsync, cuMemAlloc, ...)
 * from the TLSF pool of libptx_core.so.
 *
 * Replaces native/core/include/ptx_hook.h:14-21 (thread-mode constants and
 * ptx_hook_set/get_thread_mode, same values and meaning).
 * ptx_hook_get_stats and ptx_hook_get_runtime are additive.
 *
 * Environment (read once, when the library loads or on the first
 * allocation):
 *   PTX_HOOK_MODE=tlsf|cuda|hybrid  where allocations go (default tlsf)
 *   PTX_HOOK_HYBRID_FALLBACK=1      hybrid: a TLSF failure falls back to CUDA
 *   PTX_HOOK_DISABLE=1              no pool: TLSF-routed allocations fail
 *   PTX_HOOK_DEVICE=n               device of the pool (default 0)
 *   PTX_RUNTIME_PTR=<hex>           use this GPUHotRuntime* instead of making one
 *   PTX_HOOK_VERBOSE=1              log each routed call to stderr
 *   PTX_POOL_SIZE=<bytes>           pool size (read by gpu_hot_init)
 */
#ifndef PTX_HOOK_H
#define PTX_HOOK_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Thread-local allocator preference; only hybrid mode reads it. */
#define PTX_HOOK_THREAD_DEFAULT 0
#define PTX_HOOK_THREAD_TLSF 1
#define PTX_HOOK_THREAD_CUDA 2

void ptx_hook_set_thread_mode(int mode);
int ptx_hook_get_thread_mode(void);

/* Allocations and frees served by the pool since load, and bytes handed out
 * (any pointer may be null). */
void ptx_hook_get_stats(uint64_t* allocs, uint64_t* frees, uint64_t* bytes);
/* The GPUHotRuntime* serving the pool, or null before the first routed
 * allocation (or when the pool could not be made). */
void* ptx_hook_get_runtime(void);

#ifdef __cplusplus
}
#endif

#endif /* PTX_HOOK_H */
