#pragma once
// One sequence's logical-block -> physical-page map (reference:
// include/kvflux/v2/block_table.h:14-61). Entry i is logical block i; every
// entry owns one reference in the PhysicalBlockPool and gives it back on
// destruction, so the table is move-only.
//
// Beyond the reference's interface the table tracks its own changes, so that
// a consumer keeping a copy of the ids (the device-resident page table of
// paged_attention_batch) can refresh only what changed: lineage() names the
// table's contents and is new after construction and after a move (both
// ends), revision() is new after every edit that is not an append, and
// first_changed_since() says from which entry on a copy taken at an earlier
// revision may be out of date.
#include "kvflux/physical_block_pool.h"

#include <array>
#include <cstddef>
#include <cstdint>
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
    // out[j - first] = physical_id(j) for entries j in [first, size()) (the
    // same checks and exceptions, in entry order), with the pool's
    // bookkeeping of entry j + 32 prefetched while entry j is checked:
    // entries are random pages, so one lookup after another would wait on a
    // cache miss each.
    void copy_ids(PhysicalBlockID* out, std::size_t first = 0) const;

    // Change tracking (see the file comment). Stamps come from one
    // process-wide counter, so equal values always mean the same contents.
    std::uint64_t lineage() const noexcept { return lineage_; }
    std::uint64_t revision() const noexcept { return revision_; }
    // Lowest entry index that may differ from what it held when revision()
    // returned `revision` (an earlier value of this lineage): size() when
    // only appends happened since, 0 when `revision` is too old to tell.
    std::size_t first_changed_since(std::uint64_t revision) const noexcept;
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
    // Records an edit of entries from `index` on (not an append).
    void edited(std::size_t index) noexcept;

    struct Edit {
        std::uint64_t stamp;  // revision() after the edit
        std::size_t index;    // lowest entry it touched
    };
    static constexpr std::size_t kEdits = 4;

    PhysicalBlockPool* pool_;  // null after being moved from
    std::vector<PhysicalBlockHandle> entries_;
    std::uint64_t lineage_;
    std::uint64_t revision_;
    std::array<Edit, kEdits> edits_{};  // ring of the latest edits
    std::uint64_t edit_count_ = 0;      // edits since the lineage began
};

inline PhysicalBlockID BlockTable::physical_id(std::size_t logical_block) const {
    return pool_->id(entries_.at(logical_block));  // generation-checked
}

inline void BlockTable::copy_ids(PhysicalBlockID* out, std::size_t first) const {
    constexpr std::size_t kAhead = 32;
    const std::size_t n = entries_.size();
    for (std::size_t j = first; j < n && j < first + kAhead; ++j) pool_->prefetch(entries_[j]);
    for (std::size_t j = first; j < n; ++j) {
        if (j + kAhead < n) pool_->prefetch(entries_[j + kAhead]);
        out[j - first] = pool_->id(entries_[j]);  // generation-checked
    }
}

} // namespace kvflux::v2
