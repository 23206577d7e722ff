// Per-request token count and page growth, fork and copy-on-write
// (reference: src/v2/sequence_state.cpp:9-113).
#include "kvflux/v2/sequence_state.h"

#include <limits>
#include <stdexcept>
#include <utility>

namespace kvflux::v2 {

SequenceState::SequenceState(RequestID request_id, PhysicalBlockPool& pool) noexcept
    : request_id_(request_id), block_size_(pool.block_size()), table_(pool) {}

SequenceState::SequenceState(SequenceState&& other) noexcept
    : request_id_(other.request_id_),
      num_tokens_(std::exchange(other.num_tokens_, 0)),
      block_size_(other.block_size_),
      table_(std::move(other.table_)) {}

SequenceState& SequenceState::operator=(SequenceState&& other) noexcept {
    if (this != &other) {
        table_ = std::move(other.table_);
        request_id_ = other.request_id_;
        num_tokens_ = std::exchange(other.num_tokens_, 0);
        block_size_ = other.block_size_;
    }
    return *this;
}

std::size_t SequenceState::last_block_num_tokens() const noexcept {
    if (num_tokens_ == 0) return 0;
    const std::size_t r = num_tokens_ % block_size_;
    return r == 0 ? block_size_ : r;
}

void SequenceState::append_tokens(std::size_t count) {
    if (count == 0) return;
    if (count > std::numeric_limits<std::size_t>::max() - num_tokens_) {
        throw std::overflow_error("sequence token count would overflow");
    }
    if (num_tokens_ % block_size_ != 0 && table_.ref_count(table_.size() - 1) > 1) {
        throw std::logic_error("last page is shared and partial: append needs copy-on-write");
    }
    const std::size_t total = num_tokens_ + count;
    const std::size_t pages = total / block_size_ + (total % block_size_ != 0);
    const std::size_t before = table_.size();
    try {
        while (table_.size() < pages) table_.append_new();
    } catch (...) {
        while (table_.size() > before) table_.pop_back();
        throw;
    }
    num_tokens_ = total;
}

TokenLocation SequenceState::append_token() {
    const std::size_t position = num_tokens_;
    append_tokens(1);
    return token_location(position);
}

SequenceState SequenceState::fork_shared(RequestID new_request_id) const {
    SequenceState child(new_request_id, table_.pool());
    // If a retain throws, child's destructor frees what it already holds.
    for (std::size_t i = 0; i < table_.size(); ++i) child.table_.append_shared(table_, i);
    child.num_tokens_ = num_tokens_;
    return child;
}

TokenLocation SequenceState::append_token_with_copy(const BlockCopier& copy) {
    if (num_tokens_ == std::numeric_limits<std::size_t>::max()) {
        throw std::overflow_error("sequence token count would overflow");
    }
    const std::size_t offset = num_tokens_ % block_size_;
    if (offset == 0 || table_.ref_count(table_.size() - 1) == 1) return append_token();
    if (!copy) throw std::invalid_argument("a page copier is required for a shared partial page");

    const PhysicalBlockHandle shared = table_.handle(table_.size() - 1);
    PhysicalBlockPool& pool = table_.pool();
    const PhysicalBlockHandle fresh = pool.allocate();
    try {
        copy(shared, fresh);  // mapping and count stay untouched until it succeeds
        table_.replace_last_owned(fresh);
    } catch (...) {
        pool.free(fresh);
        throw;
    }
    ++num_tokens_;
    return {fresh.id, offset};
}

void SequenceState::append_cached_full_block(PhysicalBlockHandle h) {
    if (num_tokens_ % block_size_ != 0 ||
        block_size_ > std::numeric_limits<std::size_t>::max() - num_tokens_) {
        throw std::invalid_argument("a cached page needs a whole-page prefix before it");
    }
    table_.append_existing(h);
    num_tokens_ += block_size_;
}

void SequenceState::drop_last_full_block() noexcept {
    if (table_.empty()) return;
    try {
        table_.pop_back();
    } catch (...) {
    }
    num_tokens_ = num_tokens_ >= block_size_ ? num_tokens_ - block_size_ : 0;
}

PhysicalBlockHandle SequenceState::block_handle(std::size_t logical_block) const {
    return table_.handle(logical_block);
}

TokenLocation SequenceState::token_location(std::size_t token_index) const {
    if (token_index >= num_tokens_) throw std::out_of_range("token index beyond the sequence");
    return {physical_block_id(token_index / block_size_), token_index % block_size_};
}

} // namespace kvflux::v2
