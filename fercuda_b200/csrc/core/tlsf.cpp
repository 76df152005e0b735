#include "tlsf.hpp"

#include <cstdio>
#include <cstring>

namespace fer::pool {

// ---------------------------------------------------------------- OffsetTable

void OffsetTable::rehash(size_t cap) {
    std::vector<Slot> old;
    old.swap(slots_);
    slots_.assign(cap, Slot{0, 0});
    mask_ = cap - 1;
    shift_ = 64 - __builtin_ctzll(cap);
    count_ = 0;
    for (const Slot& s : old)
        if (s.key) insert(s.key - 1, s.val);
}

void OffsetTable::insert(uint64_t off, uint32_t idx) {
    if ((count_ + 1) * 2 > slots_.size()) rehash(slots_.size() * 2);
    const uint64_t key = off + 1;
    size_t i = slot_of(key);
    while (slots_[i].key != 0) {
        if (slots_[i].key == key) { slots_[i].val = idx; return; }
        i = (i + 1) & mask_;
    }
    slots_[i] = Slot{key, idx};
    ++count_;
}

uint32_t OffsetTable::find(uint64_t off) const {
    const uint64_t key = off + 1;
    size_t i = slot_of(key);
    while (slots_[i].key != 0) {
        if (slots_[i].key == key) return slots_[i].val;
        i = (i + 1) & mask_;
    }
    return kNil;
}

bool OffsetTable::erase(uint64_t off) {
    const uint64_t key = off + 1;
    size_t i = slot_of(key);
    while (slots_[i].key != key) {
        if (slots_[i].key == 0) return false;
        i = (i + 1) & mask_;
    }
    // Backward-shift deletion: pull later members of the probe run into the
    // hole so that no tombstones are needed.
    size_t hole = i;
    size_t j = (i + 1) & mask_;
    while (slots_[j].key != 0) {
        const size_t home = slot_of(slots_[j].key);
        // Move j into the hole if its home is not in (hole, j] cyclically.
        const bool between = (hole <= j) ? (home > hole && home <= j) : (home > hole || home <= j);
        if (!between) {
            slots_[hole] = slots_[j];
            hole = j;
        }
        j = (j + 1) & mask_;
    }
    slots_[hole] = Slot{0, 0};
    --count_;
    return true;
}

// ----------------------------------------------------------------------- Tlsf

void Tlsf::mapping(uint64_t size, int* fl, int* sl) {
    if (size < kMinBlock) { *fl = 0; *sl = 0; return; }
    int f = 63 - __builtin_clzll(size);
    if (f >= kFL) f = kFL - 1;
    *fl = f;
    *sl = (f >= 4) ? static_cast<int>((size >> (f - 4)) & (kSL - 1)) : 0;
}

Tlsf::Tlsf(uint64_t pool_size) : pool_size_(pool_size) {
    for (auto& row : heads_)
        for (auto& h : row) h = kNil;
    blocks_.reserve(1024);
    const uint32_t b = new_block();
    blocks_[b].off = 0;
    blocks_[b].size = pool_size;
    first_ = b;
    c_.total_blocks = 1;
    push_free(b);
}

uint32_t Tlsf::new_block() {
    uint32_t idx;
    if (!spare_.empty()) {
        idx = spare_.back();
        spare_.pop_back();
        blocks_[idx] = Block{};
    } else {
        idx = static_cast<uint32_t>(blocks_.size());
        blocks_.emplace_back();
    }
    return idx;
}

void Tlsf::drop_block(uint32_t idx) { spare_.push_back(idx); }

void Tlsf::push_free(uint32_t idx) {
    Block& b = blocks_[idx];
    int fl, sl;
    mapping(b.size, &fl, &sl);
    b.prev_free = kNil;
    b.next_free = heads_[fl][sl];
    if (b.next_free != kNil) blocks_[b.next_free].prev_free = idx;
    heads_[fl][sl] = idx;
    sl_bits_[fl] |= 1u << sl;
    fl_bits_ |= 1ull << fl;
    b.is_free = 1;
    ++c_.free_blocks;
    ++c_.free_list_counts[fl];
}

void Tlsf::unlink_free(uint32_t idx) {
    Block& b = blocks_[idx];
    int fl, sl;
    mapping(b.size, &fl, &sl);
    if (b.prev_free != kNil) blocks_[b.prev_free].next_free = b.next_free;
    else heads_[fl][sl] = b.next_free;
    if (b.next_free != kNil) blocks_[b.next_free].prev_free = b.prev_free;
    if (heads_[fl][sl] == kNil) {
        sl_bits_[fl] &= ~(1u << sl);
        if (!sl_bits_[fl]) fl_bits_ &= ~(1ull << fl);
    }
    b.prev_free = b.next_free = kNil;
    b.is_free = 0;
    --c_.free_blocks;
    --c_.free_list_counts[fl];
}

uint32_t Tlsf::find_fit(uint64_t size) const {
    int fl, sl;
    mapping(size, &fl, &sl);
    if (fl == kFL - 1) {
        // Clamped top class: list members are not ordered by sl, so every
        // head from sl upward is checked (the reference does the same).
        for (int s = sl; s < kSL; ++s) {
            const uint32_t h = heads_[fl][s];
            if (h != kNil && blocks_[h].size >= size) return h;
        }
        return kNil;
    }
    const uint32_t h = heads_[fl][sl];
    if (h != kNil && blocks_[h].size >= size) return h;
    // Every block of a later sl in the same fl is larger than `size`.
    const uint32_t sl_rest = sl_bits_[fl] & (~0u << (sl + 1)) & 0xFFFFu;
    if (sl_rest) return heads_[fl][__builtin_ctz(sl_rest)];
    const uint64_t fl_rest = fl_bits_ & (~0ull << (fl + 1));
    if (!fl_rest) return kNil;
    const int f = __builtin_ctzll(fl_rest);
    return heads_[f][__builtin_ctz(sl_bits_[f])];
}

uint64_t Tlsf::alloc(uint64_t size, uint32_t owner) {
    if (size == 0) return kFail;
    size = (size + kAlign - 1) & ~(kAlign - 1);
    const uint32_t idx = find_fit(size);
    if (idx == kNil) { ++c_.fallback; return kFail; }
    unlink_free(idx);
    // Split: the remainder stays free, physically after the block.
    const uint64_t rest = blocks_[idx].size - size;
    if (rest >= kMinBlock) {
        const uint32_t r = new_block();
        Block& b = blocks_[idx];
        Block& nb = blocks_[r];
        nb.off = b.off + size;
        nb.size = rest;
        nb.prev_phys = idx;
        nb.next_phys = b.next_phys;
        if (b.next_phys != kNil) blocks_[b.next_phys].prev_phys = r;
        b.size = size;
        b.next_phys = r;
        push_free(r);
        ++c_.total_blocks;
        ++c_.splits;
    }
    Block& b = blocks_[idx];
    b.owner = owner;
    live_.insert(b.off, idx);
    c_.allocated_bytes += b.size;
    if (c_.allocated_bytes > c_.peak_allocated) c_.peak_allocated = c_.allocated_bytes;
    ++c_.allocated_blocks;
    ++c_.total_allocations;
    return b.off;
}

int Tlsf::free(uint64_t off) {
    uint32_t idx = live_.find(off);
    if (idx == kNil) {
        // Distinguish a double free (a free block starts here) from a bad pointer.
        return -1;
    }
    live_.erase(off);
    Block* b = &blocks_[idx];
    c_.allocated_bytes -= b->size;
    --c_.allocated_blocks;
    ++c_.total_frees;
    b->owner = 0;
    // Merge with the next physical block.
    const uint32_t nx = b->next_phys;
    if (nx != kNil && blocks_[nx].is_free && !blocks_[nx].pinned) {
        unlink_free(nx);
        b->size += blocks_[nx].size;
        b->next_phys = blocks_[nx].next_phys;
        if (b->next_phys != kNil) blocks_[b->next_phys].prev_phys = idx;
        drop_block(nx);
        b = &blocks_[idx];
        --c_.total_blocks;
        ++c_.merges;
    }
    // Merge into the previous physical block.
    const uint32_t pv = b->prev_phys;
    if (pv != kNil && blocks_[pv].is_free && !blocks_[pv].pinned) {
        unlink_free(pv);
        Block& p = blocks_[pv];
        p.size += b->size;
        p.next_phys = b->next_phys;
        if (p.next_phys != kNil) blocks_[p.next_phys].prev_phys = pv;
        drop_block(idx);
        idx = pv;
        --c_.total_blocks;
        ++c_.merges;
    }
    push_free(idx);
    return 0;
}

uint64_t Tlsf::block_size(uint64_t off) const {
    const uint32_t idx = live_.find(off);
    return idx == kNil ? 0 : blocks_[idx].size;
}

bool Tlsf::block_info(uint64_t off, uint64_t* size, bool* is_free) const {
    uint32_t idx = live_.find(off);
    if (idx == kNil) {
        // Free blocks are not indexed; walk the chain (diagnostic path).
        for (uint32_t i = first_; i != kNil; i = blocks_[i].next_phys)
            if (blocks_[i].off == off) { idx = i; break; }
        if (idx == kNil) return false;
    }
    if (size) *size = blocks_[idx].size;
    if (is_free) *is_free = blocks_[idx].is_free != 0;
    return true;
}

bool Tlsf::set_pinned(uint64_t off, bool pinned) {
    const uint32_t idx = live_.find(off);
    if (idx == kNil) return false;
    blocks_[idx].pinned = pinned ? 1 : 0;
    return true;
}

uint32_t Tlsf::free_owner(uint32_t owner) {
    if (owner == 0) return 0;
    std::vector<uint64_t> offs;
    for (uint32_t i = first_; i != kNil; i = blocks_[i].next_phys)
        if (!blocks_[i].is_free && blocks_[i].owner == owner) offs.push_back(blocks_[i].off);
    for (uint64_t o : offs) free(o);
    return static_cast<uint32_t>(offs.size());
}

bool Tlsf::can_allocate(uint64_t size) const {
    if (size == 0) return false;
    size = (size + kAlign - 1) & ~(kAlign - 1);
    return find_fit(size) != kNil;
}

uint64_t Tlsf::largest_free() const {
    uint64_t best = 0;
    if (!fl_bits_) return 0;
    const int f = 63 - __builtin_clzll(fl_bits_);
    // Only the top non-empty first level can hold the largest block; within
    // the clamped top level lists are unordered, so scan all of them.
    for (int s = 0; s < kSL; ++s)
        for (uint32_t i = heads_[f][s]; i != kNil; i = blocks_[i].next_free)
            if (blocks_[i].size > best) best = blocks_[i].size;
    return best;
}

uint64_t Tlsf::smallest_free() const {
    uint64_t best = 0;
    if (!fl_bits_) return 0;
    const int f = __builtin_ctzll(fl_bits_);
    for (int s = 0; s < kSL; ++s)
        for (uint32_t i = heads_[f][s]; i != kNil; i = blocks_[i].next_free)
            if (best == 0 || blocks_[i].size < best) best = blocks_[i].size;
    return best;
}

void Tlsf::reset_counters() {
    const Counters keep = c_;
    c_ = Counters{};
    c_.allocated_bytes = keep.allocated_bytes;
    c_.peak_allocated = keep.allocated_bytes;
    c_.allocated_blocks = keep.allocated_blocks;
    c_.free_blocks = keep.free_blocks;
    c_.total_blocks = keep.total_blocks;
    std::memcpy(c_.free_list_counts, keep.free_list_counts, sizeof(c_.free_list_counts));
}

int Tlsf::validate(char (*msgs)[256], int max_msgs) const {
    int errs = 0;
    auto report = [&](const char* m, unsigned long long a, unsigned long long b) {
        if (msgs && errs < max_msgs) std::snprintf(msgs[errs], 256, m, a, b);
        ++errs;
    };
    uint64_t expect_off = 0, free_bytes = 0, used_bytes = 0;
    uint32_t nblocks = 0, nfree = 0, nused = 0;
    uint32_t prev = kNil;
    bool prev_free = false;
    for (uint32_t i = first_; i != kNil; i = blocks_[i].next_phys) {
        const Block& b = blocks_[i];
        if (b.off != expect_off) report("block at offset %llu, expected %llu", b.off, expect_off);
        if (b.prev_phys != prev) report("broken prev link at offset %llu (block %llu)", b.off, i);
        if (b.size == 0) report("zero-size block at offset %llu%llu", b.off, 0);
        if (b.is_free && prev_free && !b.pinned) report("adjacent free blocks at offset %llu%llu", b.off, 0);
        if (b.is_free) { free_bytes += b.size; ++nfree; }
        else {
            used_bytes += b.size; ++nused;
            if (live_.find(b.off) != i) report("allocated block at offset %llu missing from index%llu", b.off, 0);
        }
        prev_free = b.is_free && !b.pinned;
        expect_off = b.off + b.size;
        prev = i;
        ++nblocks;
        if (nblocks > blocks_.size()) { report("cycle in physical chain%llu%llu", 0, 0); break; }
    }
    if (expect_off != pool_size_) report("chain covers %llu of %llu bytes", expect_off, pool_size_);
    if (used_bytes != c_.allocated_bytes) report("allocated bytes %llu != counter %llu", used_bytes, c_.allocated_bytes);
    if (nfree != c_.free_blocks) report("free blocks %llu != counter %llu", nfree, c_.free_blocks);
    if (nused != live_.size()) report("allocated blocks %llu != index size %llu", nused, live_.size());
    // Free lists: every member is free and sits in its size class.
    uint32_t listed = 0;
    for (int f = 0; f < kFL; ++f)
        for (int s = 0; s < kSL; ++s) {
            const bool bit = (sl_bits_[f] >> s) & 1u;
            if (bit != (heads_[f][s] != kNil)) report("bitmap mismatch at fl %llu sl %llu", f, s);
            for (uint32_t i = heads_[f][s]; i != kNil; i = blocks_[i].next_free) {
                int ff, ss;
                mapping(blocks_[i].size, &ff, &ss);
                if (ff != f || ss != s) report("block at offset %llu in wrong list (fl %llu)", blocks_[i].off, f);
                if (!blocks_[i].is_free) report("allocated block at offset %llu on a free list%llu", blocks_[i].off, 0);
                if (++listed > blocks_.size()) { report("cycle in free list fl %llu sl %llu", f, s); break; }
            }
        }
    if (listed != nfree) report("free-listed %llu != free blocks %llu", listed, nfree);
    (void)free_bytes;
    return errs;
}

}  // namespace fer::pool
