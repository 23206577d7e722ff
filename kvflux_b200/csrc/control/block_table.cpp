// Logical -> physical page table with owned references and change tracking.
//
// Observable behaviour is the reference's (src/v2/block_table.cpp:8-101):
// every entry holds one pool reference, appends are all-or-nothing, lookups
// re-check the handle's generation, replace_last_owned takes over a private
// unpublished page, moves hand the references over. What is added is the
// change record that lets a copy of the ids elsewhere (a device-resident batch
// table) be refreshed by re-reading only the entries that changed: appends
// leave revision() alone, every other edit takes a new stamp from one
// process-wide counter and is remembered (stamp, lowest index touched) in a
// ring of the last kEdits edits.
#include "kvflux/v2/block_table.h"

#include <atomic>
#include <stdexcept>
#include <utility>

namespace kvflux::v2 {
namespace {

std::uint64_t next_stamp() noexcept {
    static std::atomic<std::uint64_t> counter{0};
    return counter.fetch_add(1, std::memory_order_relaxed) + 1;
}

}  // namespace

BlockTable::BlockTable(PhysicalBlockPool& pool) noexcept
    : pool_(&pool), lineage_(next_stamp()), revision_(lineage_) {}

BlockTable::~BlockTable() noexcept { clear(); }

BlockTable::BlockTable(BlockTable&& other) noexcept
    : pool_(std::exchange(other.pool_, nullptr)),
      entries_(std::move(other.entries_)),
      lineage_(next_stamp()),
      revision_(lineage_) {
    other.entries_.clear();
    other.lineage_ = other.revision_ = next_stamp();
    other.edit_count_ = 0;
}

BlockTable& BlockTable::operator=(BlockTable&& other) noexcept {
    if (this != &other) {
        clear();  // give back what this table held before taking the other's
        pool_ = std::exchange(other.pool_, nullptr);
        entries_ = std::move(other.entries_);
        other.entries_.clear();
        lineage_ = revision_ = next_stamp();
        edit_count_ = 0;
        other.lineage_ = other.revision_ = next_stamp();
        other.edit_count_ = 0;
    }
    return *this;
}

void BlockTable::edited(std::size_t index) noexcept {
    revision_ = next_stamp();
    edits_[edit_count_ % kEdits] = Edit{revision_, index};
    ++edit_count_;
}

std::size_t BlockTable::first_changed_since(std::uint64_t revision) const noexcept {
    if (revision == revision_) return entries_.size();
    // Edits after `revision` are the recorded ones with a larger stamp; they
    // are all still in the ring unless more than kEdits happened since.
    const std::uint64_t kept = edit_count_ < kEdits ? edit_count_ : kEdits;
    std::size_t low = entries_.size();
    bool reached = edit_count_ <= kEdits;  // nothing was ever dropped
    for (std::uint64_t i = 0; i < kept; ++i) {
        const Edit& e = edits_[(edit_count_ - 1 - i) % kEdits];
        if (e.stamp <= revision) {
            reached = true;
            break;
        }
        if (e.index < low) low = e.index;
    }
    if (!reached || revision < lineage_) return 0;
    return low;
}

PhysicalBlockPool& BlockTable::pool() const {
    if (pool_ == nullptr) throw std::logic_error("block table was moved from");
    return *pool_;
}

PhysicalBlockID BlockTable::append_new() {
    PhysicalBlockPool& p = pool();
    entries_.reserve(entries_.size() + 1);  // the push below cannot throw
    const PhysicalBlockHandle h = p.allocate();
    entries_.push_back(h);
    return h.id;
}

void BlockTable::append_existing(PhysicalBlockHandle h) {
    PhysicalBlockPool& p = pool();
    entries_.reserve(entries_.size() + 1);
    p.retain(h);
    entries_.push_back(h);
}

void BlockTable::append_shared(const BlockTable& source, std::size_t logical_block) {
    if (pool_ == nullptr || source.pool_ != pool_) {
        throw std::invalid_argument("shared block must come from the same physical pool");
    }
    // Read the handle before append_existing may grow (and move) entries_:
    // source may be this table.
    const PhysicalBlockHandle h = source.entries_.at(logical_block);
    append_existing(h);
}

PhysicalBlockHandle BlockTable::handle(std::size_t logical_block) const {
    const PhysicalBlockHandle h = entries_.at(logical_block);
    (void)pool_->id(h);
    return h;
}

std::size_t BlockTable::ref_count(std::size_t logical_block) const {
    return pool_->ref_count(entries_.at(logical_block));
}

void BlockTable::pop_back() {
    if (entries_.empty()) throw std::out_of_range("pop_back on an empty block table");
    pool_->free(entries_.back());
    entries_.pop_back();
    edited(entries_.size());
}

void BlockTable::replace_last_owned(PhysicalBlockHandle new_handle) {
    if (entries_.empty()) throw std::out_of_range("replace_last_owned on an empty block table");
    (void)pool_->id(new_handle);
    if (new_handle == entries_.back() || pool_->ref_count(new_handle) != 1 ||
        pool_->is_published(new_handle)) {
        throw std::invalid_argument("replacement page must be private and unpublished");
    }
    // free() validates the old handle before anything changes; the assignment
    // after it cannot throw, so a failure leaves the caller owning new_handle.
    pool_->free(entries_.back());
    entries_.back() = new_handle;
    edited(entries_.size() - 1);
}

void BlockTable::clear() noexcept {
    if (entries_.empty()) return;
    if (pool_ != nullptr) {
        for (const PhysicalBlockHandle& h : entries_) pool_->free(h);
    }
    entries_.clear();
    edited(0);
}

}  // namespace kvflux::v2
