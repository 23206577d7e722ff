#pragma once
// Per-request token count and page ownership (reference:
// include/kvflux/v2/sequence_state.h:21-71). Holds no K/V data.
#include "kvflux/v2/block_table.h"

#include <cstddef>
#include <cstdint>
#include <functional>

namespace kvflux::v2 {

using RequestID = std::uint64_t;
class PrefixCache;

struct TokenLocation {
    PhysicalBlockID physical_block;
    std::size_t offset_in_block;
};

class SequenceState {
public:
    SequenceState(RequestID request_id, PhysicalBlockPool& pool) noexcept;

    SequenceState(const SequenceState&) = delete;
    SequenceState& operator=(const SequenceState&) = delete;
    SequenceState(SequenceState&& other) noexcept;
    SequenceState& operator=(SequenceState&& other) noexcept;

    RequestID request_id() const noexcept { return request_id_; }
    std::size_t num_tokens() const noexcept { return num_tokens_; }
    std::size_t block_size() const noexcept { return block_size_; }
    const BlockTable& block_table() const noexcept { return table_; }
    std::size_t num_allocated_blocks() const noexcept { return table_.size(); }
    // 0 for an empty sequence; a full last block reports block_size, not 0.
    std::size_t last_block_num_tokens() const noexcept;

    // Reserves positions (and pages) for `count` more tokens. All-or-nothing.
    // Refuses to grow into a shared partial last page (logic_error).
    void append_tokens(std::size_t count);
    TokenLocation append_token();

    // New request sharing every page of this one (each entry retained).
    SequenceState fork_shared(RequestID new_request_id) const;

    using BlockCopier = std::function<void(PhysicalBlockHandle source,
                                           PhysicalBlockHandle destination)>;
    // Decode append with copy-on-write of a shared partial last page.
    TokenLocation append_token_with_copy(const BlockCopier& copy);

    PhysicalBlockID physical_block_id(std::size_t logical_block) const;
    // out[j] = physical_block_id(j) for j < num_allocated_blocks(), in one
    // pass (BlockTable::copy_ids).
    void copy_physical_block_ids(PhysicalBlockID* out) const { table_.copy_ids(out); }
    TokenLocation token_location(std::size_t token_index) const;

private:
    friend class PrefixCache;
    void append_cached_full_block(PhysicalBlockHandle handle);
    PhysicalBlockHandle block_handle(std::size_t logical_block) const;
    void drop_last_full_block() noexcept;

    RequestID request_id_;
    std::size_t num_tokens_ = 0;
    std::size_t block_size_;
    BlockTable table_;
};

inline PhysicalBlockID SequenceState::physical_block_id(std::size_t logical_block) const {
    return table_.physical_id(logical_block);
}

} // namespace kvflux::v2
