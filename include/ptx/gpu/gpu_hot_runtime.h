/*
 * Native memory-runtime ABI (libptx_core.so): the TLSF-backed device pool
 * that every fercuda buffer is served from.
 *
 * Replaces the subset of the reference native/core/include/gpu/gpu_hot_runtime.h
 * that the hot path uses:
 *   - TLSF constants            gpu_hot_runtime.h:35-38
 *   - TLSFPoolStats             gpu_hot_runtime.h:384-419
 *   - TLSFOwnerUsage/Stats      gpu_hot_runtime.h:422-432
 *   - TLSFAllocEvent/EventRing  gpu_hot_runtime.h:439-454
 *   - TLSFHealthReport          gpu_hot_runtime.h:460-468
 *   - GPUHotConfig              gpu_hot_runtime.h:490-520
 *   - gpu_hot_* pool entry points gpu_hot_runtime.h:522-545
 * Struct layouts match the reference so existing callers of these entry
 * points link unchanged. GPUHotRuntime is opaque. The reference's process
 * registry, watchdog, VMM/VFS, task queue and NVML/CUPTI polling are not part
 * of this library.
 */
#ifndef FERCUDA_PTX_GPU_HOT_RUNTIME_H
#define FERCUDA_PTX_GPU_HOT_RUNTIME_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TLSF_FL_INDEX_MAX   34
#define TLSF_SL_INDEX_COUNT 16
#define TLSF_MIN_BLOCK_SIZE 64
#define TLSF_ALIGNMENT      256

typedef struct TLSFPoolStats {
    size_t total_pool_size;
    size_t allocated_bytes;
    size_t free_bytes;
    size_t peak_allocated;
    size_t largest_free_block;
    size_t smallest_free_block;

    uint32_t total_blocks;
    uint32_t free_blocks;
    uint32_t allocated_blocks;

    uint32_t fallback_count;
    float utilization_percent;
    float fragmentation_ratio;
    float external_fragmentation;

    uint32_t free_list_counts[34];

    uint32_t hash_collisions;
    uint32_t max_chain_length;
    float avg_chain_length;

    uint64_t total_allocations;
    uint64_t total_frees;
    uint32_t total_splits;
    uint32_t total_merges;

    bool is_healthy;
    bool needs_defrag;
} TLSFPoolStats;

#define TLSF_MAX_OWNERS 64

typedef struct TLSFOwnerUsage {
    uint32_t owner_id;
    size_t allocated_bytes;
    uint32_t block_count;
} TLSFOwnerUsage;

typedef struct TLSFOwnerStats {
    TLSFOwnerUsage owners[TLSF_MAX_OWNERS];
    uint32_t num_owners;
} TLSFOwnerStats;

#define TLSF_EVENT_RING_SIZE 256

typedef struct TLSFAllocEvent {
    uint64_t timestamp;
    size_t size;
    uint32_t owner_id;
    uint32_t alloc_id;
    uint8_t event_type;   /* 0 alloc, 1 free, 2 realloc */
    uint8_t _pad[3];
} TLSFAllocEvent;

typedef struct TLSFEventRing {
    TLSFAllocEvent events[TLSF_EVENT_RING_SIZE];
    uint32_t head;
    uint32_t count;
} TLSFEventRing;

typedef struct TLSFHealthReport {
    bool is_valid;
    bool has_memory_leaks;
    bool has_corrupted_blocks;
    bool has_broken_chains;
    bool has_hash_errors;
    int error_count;
    char error_messages[16][256];
} TLSFHealthReport;

typedef struct GPUHotConfig {
    float pool_fraction;        /* fraction of free VRAM; 0 = use fixed_pool_size */
    size_t fixed_pool_size;
    size_t min_pool_size;
    size_t max_pool_size;
    size_t reserve_vram;
    bool enable_leak_detection;
    bool enable_pool_health;
    float warning_threshold;
    bool force_daemon_mode;     /* accepted, no effect */
    bool quiet_init;
    unsigned int max_streams;
    bool single_pool_strict;    /* accepted, no effect */
} GPUHotConfig;

typedef struct GPUHotRuntime GPUHotRuntime;

GPUHotConfig gpu_hot_default_config(void);
GPUHotRuntime* gpu_hot_init(int device_id, const char* token);
GPUHotRuntime* gpu_hot_init_with_config(int device_id, const char* token, const GPUHotConfig* config);
void gpu_hot_shutdown(GPUHotRuntime* runtime);

void* gpu_hot_alloc(GPUHotRuntime* runtime, size_t size);
void gpu_hot_free(GPUHotRuntime* runtime, void* ptr);
/* Stream-ordered variants: the free becomes effective once all work queued
 * on `stream` before the call has completed. */
void* gpu_hot_alloc_async(GPUHotRuntime* runtime, size_t size, cudaStream_t stream);
void gpu_hot_free_async(GPUHotRuntime* runtime, void* ptr, cudaStream_t stream);
void gpu_hot_poll_deferred(GPUHotRuntime* runtime, int max_drain);
bool gpu_hot_can_allocate(GPUHotRuntime* runtime, size_t size);
size_t gpu_hot_get_max_allocatable(GPUHotRuntime* runtime);
bool gpu_hot_owns_ptr(GPUHotRuntime* runtime, void* ptr);
void* gpu_hot_alloc_owned(GPUHotRuntime* runtime, size_t size, uint32_t owner_id);
void gpu_hot_free_owner(GPUHotRuntime* runtime, uint32_t owner_id);
void gpu_hot_get_owner_stats(GPUHotRuntime* runtime, TLSFOwnerStats* stats);
void gpu_hot_get_alloc_events(GPUHotRuntime* runtime, TLSFEventRing* ring_out);
/* Stream `index` of the runtime's stream set (index 0 is the session stream). */
cudaStream_t gpu_hot_get_stream(GPUHotRuntime* runtime, int index);
void gpu_hot_get_tlsf_stats(GPUHotRuntime* runtime, TLSFPoolStats* stats);
void gpu_hot_validate_tlsf_pool(GPUHotRuntime* runtime, TLSFHealthReport* report);

#ifdef __cplusplus
}
#endif

#endif
