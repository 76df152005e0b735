// C entry points of the TLSF allocator (ptx_tlsf_*), over fer::pool::Tlsf.
//
// Replaces the reference native/core/memory/tlsf_allocator.cu public API
// (modules/tlsf_allocator_api.inl:9-832). Bookkeeping is host-only; only
// ptx_tlsf_create / ptx_tlsf_destroy touch the device (one cudaMalloc /
// cudaFree for an owned pool).
#include "memory/ptx_tlsf_allocator.h"

#include "tlsf.hpp"

#include <cuda_runtime_api.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <ctime>
#include <new>
#include <unordered_map>

struct PTXTLSFAllocator {
    uintptr_t base = 0;
    bool owns = false;
    bool debug = false;
    bool warnings = true;
    float warning_threshold = 0.8f;
    fer::pool::Tlsf tlsf;
    TLSFEventRing ring{};
    PTXTLSFAllocator(uintptr_t b, uint64_t size) : base(b), tlsf(size) {}
};

namespace {

uint64_t now_us() {
    timespec ts;
    clock_gettime(CLOCK_MONOTONIC_COARSE, &ts);
    return static_cast<uint64_t>(ts.tv_sec) * 1000000ull + static_cast<uint64_t>(ts.tv_nsec) / 1000ull;
}

void push_event(PTXTLSFAllocator* a, uint64_t size, uint32_t owner, uint8_t type) {
    TLSFAllocEvent& ev = a->ring.events[a->ring.head % TLSF_EVENT_RING_SIZE];
    ev.timestamp = now_us();
    ev.size = size;
    ev.owner_id = owner;
    ev.alloc_id = static_cast<uint32_t>(a->tlsf.counters().total_allocations);
    ev.event_type = type;
    a->ring.head++;
    a->ring.count++;
}

bool in_pool(const PTXTLSFAllocator* a, const void* p) {
    const uintptr_t u = reinterpret_cast<uintptr_t>(p);
    return u >= a->base && u < a->base + a->tlsf.pool_size();
}

void* do_alloc(PTXTLSFAllocator* a, size_t size, uint32_t owner) {
    if (!a || size == 0) return nullptr;
    const uint64_t off = a->tlsf.alloc(size, owner);
    if (off == fer::pool::Tlsf::kFail) return nullptr;
    if (a->debug) push_event(a, a->tlsf.block_size(off), owner, 0);
    return reinterpret_cast<void*>(a->base + off);
}

}  // namespace

extern "C" {

PTXTLSFAllocator* ptx_tlsf_create_from_pool(void* pool, size_t pool_size, bool debug_mode) {
    if (!pool || pool_size == 0) return nullptr;
    auto* a = new (std::nothrow) PTXTLSFAllocator(reinterpret_cast<uintptr_t>(pool), pool_size);
    if (!a) return nullptr;
    a->debug = debug_mode;
    return a;
}

PTXTLSFAllocator* ptx_tlsf_create(size_t pool_size, bool debug_mode) {
    pool_size = (pool_size + TLSF_ALIGNMENT - 1) & ~static_cast<size_t>(TLSF_ALIGNMENT - 1);
    void* pool = nullptr;
    if (pool_size == 0 || cudaMalloc(&pool, pool_size) != cudaSuccess) return nullptr;
    PTXTLSFAllocator* a = ptx_tlsf_create_from_pool(pool, pool_size, debug_mode);
    if (!a) { cudaFree(pool); return nullptr; }
    a->owns = true;
    return a;
}

void ptx_tlsf_destroy(PTXTLSFAllocator* a) {
    if (!a) return;
    if (a->owns && a->base) cudaFree(reinterpret_cast<void*>(a->base));
    delete a;
}

void* ptx_tlsf_alloc(PTXTLSFAllocator* a, size_t size) { return do_alloc(a, size, 0); }

void* ptx_tlsf_alloc_debug(PTXTLSFAllocator* a, size_t size, const char*, int) { return do_alloc(a, size, 0); }

void* ptx_tlsf_alloc_owned(PTXTLSFAllocator* a, size_t size, uint32_t owner_id) { return do_alloc(a, size, owner_id); }

void ptx_tlsf_free(PTXTLSFAllocator* a, void* ptr) {
    if (!a || !ptr || !in_pool(a, ptr)) return;
    const uint64_t off = reinterpret_cast<uintptr_t>(ptr) - a->base;
    const uint64_t sz = a->debug ? a->tlsf.block_size(off) : 0;
    if (a->tlsf.free(off) == 0 && a->debug) push_event(a, sz, 0, 1);
}

void* ptx_tlsf_realloc(PTXTLSFAllocator* a, void* ptr, size_t new_size) {
    if (!a) return nullptr;
    if (!ptr) return ptx_tlsf_alloc(a, new_size);
    if (new_size == 0) { ptx_tlsf_free(a, ptr); return nullptr; }
    if (!in_pool(a, ptr)) return nullptr;
    const uint64_t off = reinterpret_cast<uintptr_t>(ptr) - a->base;
    const uint64_t old = a->tlsf.block_size(off);
    if (old == 0) return nullptr;
    if (old >= new_size) return ptr;
    void* np = ptx_tlsf_alloc(a, new_size);
    if (!np) return nullptr;
    // Device-to-device copy of the old contents (owned or external pool alike).
    cudaMemcpy(np, ptr, old, cudaMemcpyDeviceToDevice);
    ptx_tlsf_free(a, ptr);
    return np;
}

void ptx_tlsf_free_owner(PTXTLSFAllocator* a, uint32_t owner_id) {
    if (a) a->tlsf.free_owner(owner_id);
}

void ptx_tlsf_get_owner_stats(PTXTLSFAllocator* a, TLSFOwnerStats* out) {
    if (!a || !out) return;
    std::memset(out, 0, sizeof(*out));
    a->tlsf.for_each_block([&](const fer::pool::Block& b) {
        if (b.is_free || b.owner == 0) return;
        uint32_t i = 0;
        while (i < out->num_owners && out->owners[i].owner_id != b.owner) ++i;
        if (i == out->num_owners) {
            if (out->num_owners >= TLSF_MAX_OWNERS) return;
            out->owners[i].owner_id = b.owner;
            ++out->num_owners;
        }
        out->owners[i].allocated_bytes += b.size;
        out->owners[i].block_count++;
    });
}

void ptx_tlsf_get_events(PTXTLSFAllocator* a, TLSFEventRing* out) {
    if (a && out) *out = a->ring;
}

void ptx_tlsf_get_stats(PTXTLSFAllocator* a, TLSFPoolStats* s) {
    if (!a || !s) return;
    std::memset(s, 0, sizeof(*s));
    const fer::pool::Counters& c = a->tlsf.counters();
    s->total_pool_size = a->tlsf.pool_size();
    s->allocated_bytes = c.allocated_bytes;
    s->free_bytes = a->tlsf.pool_size() - c.allocated_bytes;
    s->peak_allocated = c.peak_allocated;
    s->largest_free_block = a->tlsf.largest_free();
    s->smallest_free_block = a->tlsf.smallest_free();
    s->total_blocks = c.total_blocks;
    s->free_blocks = c.free_blocks;
    s->allocated_blocks = c.allocated_blocks;
    s->fallback_count = c.fallback;
    s->utilization_percent = 100.0f * static_cast<float>(c.allocated_bytes) / static_cast<float>(a->tlsf.pool_size());
    const double free_b = static_cast<double>(s->free_bytes);
    s->fragmentation_ratio = free_b > 0 ? static_cast<float>(1.0 - s->largest_free_block / free_b) : 0.0f;
    s->external_fragmentation = s->fragmentation_ratio;
    std::memcpy(s->free_list_counts, c.free_list_counts, sizeof(s->free_list_counts));
    s->total_allocations = c.total_allocations;
    s->total_frees = c.total_frees;
    s->total_splits = c.splits;
    s->total_merges = c.merges;
    s->max_chain_length = 1;
    s->avg_chain_length = 1.0f;
    s->is_healthy = true;
    s->needs_defrag = false;
}

void ptx_tlsf_validate(PTXTLSFAllocator* a, TLSFHealthReport* r) {
    if (!r) return;
    std::memset(r, 0, sizeof(*r));
    if (!a) { r->error_count = 1; return; }
    const int errs = a->tlsf.validate(r->error_messages, 16);
    r->error_count = errs;
    r->is_valid = errs == 0;
    r->has_broken_chains = errs != 0;
    r->has_memory_leaks = false;
}

bool ptx_tlsf_can_allocate(PTXTLSFAllocator* a, size_t size) { return a && a->tlsf.can_allocate(size); }

size_t ptx_tlsf_get_max_allocatable(PTXTLSFAllocator* a) { return a ? a->tlsf.largest_free() : 0; }

bool ptx_tlsf_owns_ptr(PTXTLSFAllocator* a, void* ptr) {
    if (!a || !ptr || !in_pool(a, ptr)) return false;
    return a->tlsf.block_size(reinterpret_cast<uintptr_t>(ptr) - a->base) != 0;
}

bool ptx_tlsf_get_block_info(PTXTLSFAllocator* a, void* ptr, size_t* size_out, bool* is_free_out) {
    if (!a || !ptr || !in_pool(a, ptr)) return false;
    uint64_t sz = 0;
    bool fr = false;
    if (!a->tlsf.block_info(reinterpret_cast<uintptr_t>(ptr) - a->base, &sz, &fr)) return false;
    if (size_out) *size_out = sz;
    if (is_free_out) *is_free_out = fr;
    return true;
}

void ptx_tlsf_pin_block(PTXTLSFAllocator* a, void* ptr) {
    if (a && ptr && in_pool(a, ptr)) a->tlsf.set_pinned(reinterpret_cast<uintptr_t>(ptr) - a->base, true);
}

void ptx_tlsf_unpin_block(PTXTLSFAllocator* a, void* ptr) {
    if (a && ptr && in_pool(a, ptr)) a->tlsf.set_pinned(reinterpret_cast<uintptr_t>(ptr) - a->base, false);
}

void ptx_tlsf_defragment(PTXTLSFAllocator*) {}
void ptx_tlsf_compact(PTXTLSFAllocator*) {}
void ptx_tlsf_reset_stats(PTXTLSFAllocator* a) { if (a) a->tlsf.reset_counters(); }
void ptx_tlsf_set_warning_threshold(PTXTLSFAllocator* a, float t) { if (a) a->warning_threshold = t; }
void ptx_tlsf_set_warnings_enabled(PTXTLSFAllocator* a, bool e) { if (a) a->warnings = e; }

}  // extern "C"
