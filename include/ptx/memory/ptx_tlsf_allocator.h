/*
 * TLSF (two-level segregated fit) allocator over one device address range.
 *
 * Entry points replace the reference native/core/include/memory/ptx_tlsf_allocator.h
 * core/alloc/diagnostic API (ptx_tlsf_allocator.h:96-175). Bookkeeping is
 * host-side; the allocator never touches device memory, so it runs unchanged
 * over a fake range on a machine without a GPU.
 *
 * Block choice is the reference's (tlsf_allocator_internals.inl:208-231):
 * the head of the request's own (fl, sl) list if it is large enough, else the
 * first non-empty list after it in (fl, sl) order. Here that search is two
 * bitmap scans instead of a loop over up to 34x16 list heads, so the same
 * trace yields the same addresses in O(1).
 */
#ifndef FERCUDA_PTX_TLSF_ALLOCATOR_H
#define FERCUDA_PTX_TLSF_ALLOCATOR_H

#include "gpu/gpu_hot_runtime.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct PTXTLSFAllocator PTXTLSFAllocator;

/* Creates a pool with its own device allocation (cudaMalloc). */
PTXTLSFAllocator* ptx_tlsf_create(size_t pool_size, bool debug_mode);
/* Manages [pool, pool+pool_size) without owning it. */
PTXTLSFAllocator* ptx_tlsf_create_from_pool(void* pool, size_t pool_size, bool debug_mode);
void ptx_tlsf_destroy(PTXTLSFAllocator* allocator);

void* ptx_tlsf_alloc(PTXTLSFAllocator* allocator, size_t size);
void* ptx_tlsf_alloc_debug(PTXTLSFAllocator* allocator, size_t size, const char* file, int line);
void ptx_tlsf_free(PTXTLSFAllocator* allocator, void* ptr);
void* ptx_tlsf_realloc(PTXTLSFAllocator* allocator, void* ptr, size_t new_size);

void* ptx_tlsf_alloc_owned(PTXTLSFAllocator* allocator, size_t size, uint32_t owner_id);
void ptx_tlsf_free_owner(PTXTLSFAllocator* allocator, uint32_t owner_id);
void ptx_tlsf_get_owner_stats(PTXTLSFAllocator* allocator, TLSFOwnerStats* stats);
void ptx_tlsf_get_events(PTXTLSFAllocator* allocator, TLSFEventRing* ring_out);

void ptx_tlsf_get_stats(PTXTLSFAllocator* allocator, TLSFPoolStats* stats);
void ptx_tlsf_validate(PTXTLSFAllocator* allocator, TLSFHealthReport* report);
bool ptx_tlsf_can_allocate(PTXTLSFAllocator* allocator, size_t size);
size_t ptx_tlsf_get_max_allocatable(PTXTLSFAllocator* allocator);
bool ptx_tlsf_owns_ptr(PTXTLSFAllocator* allocator, void* ptr);
bool ptx_tlsf_get_block_info(PTXTLSFAllocator* allocator, void* ptr, size_t* size_out, bool* is_free_out);

void ptx_tlsf_pin_block(PTXTLSFAllocator* allocator, void* ptr);
void ptx_tlsf_unpin_block(PTXTLSFAllocator* allocator, void* ptr);
/* Free blocks are coalesced eagerly, so these are consistency no-ops. */
void ptx_tlsf_defragment(PTXTLSFAllocator* allocator);
void ptx_tlsf_compact(PTXTLSFAllocator* allocator);
void ptx_tlsf_reset_stats(PTXTLSFAllocator* allocator);
void ptx_tlsf_set_warning_threshold(PTXTLSFAllocator* allocator, float threshold);
void ptx_tlsf_set_warnings_enabled(PTXTLSFAllocator* allocator, bool enabled);

#ifdef __cplusplus
}
#endif

#endif
