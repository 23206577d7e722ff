#pragma once
// Single-layer paged K/V byte layout (reference:
// include/kvflux/v2/paged_kv_layout.h:12-40):
//   K[num_blocks][num_kv_heads][block_size][head_size], then V of the same
//   shape, innermost dimension contiguous, no padding.
#include "kvflux/kv_layout.h"

#include <cstddef>
#include <cstdint>

namespace kvflux::v2 {

class PagedKVLayout {
public:
    PagedKVLayout(std::size_t num_blocks, std::size_t num_kv_heads,
                  std::size_t block_size, std::size_t head_size, DType dtype);

    std::size_t num_blocks() const noexcept { return num_blocks_; }
    std::size_t num_kv_heads() const noexcept { return num_kv_heads_; }
    std::size_t block_size() const noexcept { return block_size_; }
    std::size_t head_size() const noexcept { return head_size_; }
    DType dtype() const noexcept { return dtype_; }
    std::size_t element_bytes() const noexcept { return element_bytes_; }
    std::size_t page_bytes() const noexcept { return page_bytes_; }
    std::size_t cache_bytes() const noexcept { return cache_bytes_; }
    std::size_t total_bytes() const noexcept { return total_bytes_; }
    std::size_t slot_count() const noexcept { return slot_count_; }

    // Byte offsets from the start of the K+V allocation; all bounds-checked.
    std::size_t page_byte_offset(KVKind kind, std::size_t block) const;
    std::size_t byte_offset(KVKind kind, std::size_t block, std::size_t head,
                            std::size_t token, std::size_t dimension) const;
    std::size_t slot_byte_offset(KVKind kind, std::uint64_t slot,
                                 std::size_t head, std::size_t dimension) const;

private:
    std::size_t num_blocks_, num_kv_heads_, block_size_, head_size_;
    DType dtype_;
    std::size_t element_bytes_, page_bytes_, cache_bytes_, total_bytes_, slot_count_;
};

} // namespace kvflux::v2
