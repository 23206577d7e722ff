#pragma once
// One sequence's logical-block -> physical-page map (reference:
// include/kvflux/v2/block_table.h:14-61). Entry i is logical block i; every
// entry owns one reference in the PhysicalBlockPool and gives it back on
// destruction, so the table is move-only.
#include "kvflux/physical_block_pool.h"

#include <cstddef>
#include <vector>

namespace kvflux::v2 {

class BlockTable {
public:
    explicit BlockTable(PhysicalBlockPool& pool) noexcept;
    ~BlockTable() noexcept;

    BlockTable(const BlockTable&) = delete;
    BlockTable& operator=(const BlockTable&) = delete;
    BlockTable(BlockTable&& other) noexcept;
    BlockTable& operator=(BlockTable&& other) noexcept;

    // Allocates a fresh page and appends it; on failure the table is unchanged.
    PhysicalBlockID append_new();
    // Appends an existing page with a reference of its own (retain).
    void append_existing(PhysicalBlockHandle handle);
    // Shares logical block `logical_block` of `source` (same pool required).
    void append_shared(const BlockTable& source, std::size_t logical_block);

    // Generation-checked lookups; they add no reference.
    PhysicalBlockID physical_id(std::size_t logical_block) const;
    PhysicalBlockHandle handle(std::size_t logical_block) const;
    std::size_t ref_count(std::size_t logical_block) const;
    PhysicalBlockID operator[](std::size_t logical_block) const {
        return physical_id(logical_block);
    }
    // out[j] = physical_id(j) for every entry (the same checks and
    // exceptions, in entry order), with the pool's bookkeeping of entry
    // j + 32 prefetched while entry j is checked: entries are random pages,
    // so one lookup after another would wait on a cache miss each.
    void copy_ids(PhysicalBlockID* out) const;
    std::size_t size() const noexcept { return entries_.size(); }
    bool empty() const noexcept { return entries_.empty(); }
    bool shares_pool_with(const BlockTable& other) const noexcept {
        return pool_ != nullptr && pool_ == other.pool_;
    }
    bool uses_pool(const PhysicalBlockPool& pool) const noexcept { return pool_ == &pool; }
    PhysicalBlockPool& pool() const;

    // Drops the last entry (and its reference). Not while the GPU still reads it.
    void pop_back();
    // Takes over a caller-owned private, unpublished page as the new last entry
    // and frees the old last entry's reference. Allocates nothing.
    void replace_last_owned(PhysicalBlockHandle new_handle);
    void clear() noexcept;

private:
    PhysicalBlockPool* pool_;  // null after being moved from
    std::vector<PhysicalBlockHandle> entries_;
};

inline PhysicalBlockID BlockTable::physical_id(std::size_t logical_block) const {
    return pool_->id(entries_.at(logical_block));  // generation-checked
}

inline void BlockTable::copy_ids(PhysicalBlockID* out) const {
    constexpr std::size_t kAhead = 32;
    const std::size_t n = entries_.size();
    for (std::size_t j = 0; j < n && j < kAhead; ++j) pool_->prefetch(entries_[j]);
    for (std::size_t j = 0; j < n; ++j) {
        if (j + kAhead < n) pool_->prefetch(entries_[j + kAhead]);
        out[j] = pool_->id(entries_[j]);  // generation-checked
    }
}

} // namespace kvflux::v2
