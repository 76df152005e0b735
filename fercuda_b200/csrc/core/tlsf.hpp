// TLSF (two-level segregated fit) bookkeeping over one contiguous device
// address range. Pure host code: it hands out offsets and never touches the
// memory itself.
//
// Size classes, alignment, split and coalesce rules follow the reference
// allocator so that one alloc/free trace yields the same addresses:
//   - mapping: fl = floor(log2 size) clamped to 33, sl = next 4 bits
//     (reference native/core/memory/modules/tlsf_allocator_internals.inl:71-91)
//   - request size rounded up to 256 B (tlsf_allocator_api.inl:117)
//   - block choice: head of the request's own (fl, sl) list if large enough,
//     else the first non-empty list after it (internals.inl:208-231)
//   - split leaves the remainder (>= 64 B) after the block, pushed at the head
//     of its list (internals.inl:237-271)
//   - free merges with the next then the previous physical block, then
//     pushes the result at the head of its list (internals.inl:273-321,
//     api.inl:282-289)
// What differs is the data structure, not the decisions:
//   - the (fl, sl) search is two bitmap scans (ctz) instead of a loop over up
//     to 34x16 list heads;
//   - block headers live in a slab vector addressed by 32-bit index, with a
//     free-index stack, instead of one malloc per split;
//   - pointer -> block lookup is an open-addressed table keyed by the block's
//     offset (linear probing, backward-shift delete), grown at 50% load,
//     instead of 4096 chained buckets.
#pragma once

#include <cstddef>
#include <cstdint>
#include <vector>

namespace fer::pool {

constexpr int kFL = 34;
constexpr int kSL = 16;
constexpr uint64_t kMinBlock = 64;
constexpr uint64_t kAlign = 256;
constexpr uint32_t kNil = 0xFFFFFFFFu;

struct Block {
    uint64_t off = 0;
    uint64_t size = 0;
    uint32_t prev_phys = kNil, next_phys = kNil;
    uint32_t prev_free = kNil, next_free = kNil;
    uint32_t owner = 0;
    uint8_t is_free = 0;
    uint8_t pinned = 0;
};

struct Counters {
    uint64_t allocated_bytes = 0, peak_allocated = 0;
    uint64_t total_allocations = 0, total_frees = 0;
    uint32_t allocated_blocks = 0, free_blocks = 0, total_blocks = 0;
    uint32_t splits = 0, merges = 0, fallback = 0;
    uint32_t free_list_counts[kFL] = {};
};

// Offset -> block index map for allocated blocks.
class OffsetTable {
public:
    OffsetTable() { rehash(1024); }
    void insert(uint64_t off, uint32_t idx);
    uint32_t find(uint64_t off) const;
    bool erase(uint64_t off);
    size_t size() const { return count_; }
    void clear() { rehash(1024); }

private:
    struct Slot { uint64_t key; uint32_t val; };   // key = off + 1, 0 = empty
    void rehash(size_t cap);
    size_t slot_of(uint64_t key) const {
        return static_cast<size_t>((key * 0x9E3779B97F4A7C15ull) >> shift_);
    }
    std::vector<Slot> slots_;
    size_t mask_ = 0, count_ = 0;
    int shift_ = 64;
};

class Tlsf {
public:
    static constexpr uint64_t kFail = ~0ull;

    explicit Tlsf(uint64_t pool_size);

    // Returns the block offset, or kFail when no block fits (or size == 0).
    uint64_t alloc(uint64_t size, uint32_t owner = 0);
    // Returns 0 on success, -1 unknown offset, -2 double free.
    int free(uint64_t off);
    // Size of the allocated block at `off`, 0 if none.
    uint64_t block_size(uint64_t off) const;
    bool block_info(uint64_t off, uint64_t* size, bool* is_free) const;
    bool set_pinned(uint64_t off, bool pinned);
    // Frees every block owned by `owner`; returns how many.
    uint32_t free_owner(uint32_t owner);

    bool can_allocate(uint64_t size) const;
    uint64_t largest_free() const;
    uint64_t smallest_free() const;
    uint64_t pool_size() const { return pool_size_; }
    const Counters& counters() const { return c_; }
    void reset_counters();

    // Walks the physical chain and the free lists; returns the number of
    // inconsistencies found and writes up to `max_msgs` messages.
    int validate(char (*msgs)[256], int max_msgs) const;

    template <typename F> void for_each_block(F&& f) const {
        for (uint32_t i = first_; i != kNil; i = blocks_[i].next_phys) f(blocks_[i]);
    }

private:
    static void mapping(uint64_t size, int* fl, int* sl);
    uint32_t find_fit(uint64_t size) const;
    void push_free(uint32_t idx);
    void unlink_free(uint32_t idx);
    uint32_t new_block();
    void drop_block(uint32_t idx);

    uint64_t pool_size_;
    std::vector<Block> blocks_;
    std::vector<uint32_t> spare_;
    uint32_t heads_[kFL][kSL];
    uint64_t fl_bits_ = 0;
    uint32_t sl_bits_[kFL] = {};
    uint32_t first_ = kNil;
    OffsetTable live_;
    Counters c_;
};

}  // namespace fer::pool
