// Logical -> physical page table with owned references
// (reference: src/v2/block_table.cpp:8-101).
#include "kvflux/v2/block_table.h"

#include <stdexcept>
#include <utility>

namespace kvflux::v2 {

BlockTable::BlockTable(PhysicalBlockPool& pool) noexcept : pool_(&pool) {}

BlockTable::~BlockTable() noexcept { clear(); }

BlockTable::BlockTable(BlockTable&& other) noexcept
    : pool_(std::exchange(other.pool_, nullptr)), entries_(std::move(other.entries_)) {
    other.entries_.clear();
}

BlockTable& BlockTable::operator=(BlockTable&& other) noexcept {
    if (this != &other) {
        clear();  // give back what this table held before taking the other's
        pool_ = std::exchange(other.pool_, nullptr);
        entries_ = std::move(other.entries_);
        other.entries_.clear();
    }
    return *this;
}

PhysicalBlockPool& BlockTable::pool() const {
    if (pool_ == nullptr) throw std::logic_error("block table was moved from");
    return *pool_;
}

PhysicalBlockID BlockTable::append_new() {
    PhysicalBlockPool& p = pool();
    const PhysicalBlockHandle h = p.allocate();
    try {
        entries_.push_back(h);
    } catch (...) {
        p.free(h);
        throw;
    }
    return h.id;
}

void BlockTable::append_existing(PhysicalBlockHandle h) {
    PhysicalBlockPool& p = pool();
    p.retain(h);
    try {
        entries_.push_back(h);
    } catch (...) {
        p.free(h);
        throw;
    }
}

void BlockTable::append_shared(const BlockTable& source, std::size_t logical_block) {
    if (pool_ == nullptr || source.pool_ != pool_) {
        throw std::invalid_argument("shared block must come from the same physical pool");
    }
    // Copy the handle first: source may be *this and push_back may reallocate.
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
}

void BlockTable::clear() noexcept {
    if (pool_ != nullptr) {
        for (const PhysicalBlockHandle& h : entries_) pool_->free(h);
    }
    entries_.clear();
}

} // namespace kvflux::v2
