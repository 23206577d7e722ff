#pragma once
// Row-major [num_sequences][max_blocks_per_sequence] snapshot of a batch's
// page ids, padded with invalid_block() (reference:
// include/kvflux/v2/batch_block_table.h:12-36). It holds no page references.
#include "kvflux/v2/sequence_state.h"

#include <cstddef>
#include <vector>

namespace kvflux::v2 {

class BatchBlockTable {
public:
    std::size_t num_sequences() const noexcept { return sequence_lengths_.size(); }
    std::size_t max_blocks_per_sequence() const noexcept { return max_blocks_per_sequence_; }
    const std::vector<PhysicalBlockID>& block_table() const noexcept { return block_table_; }
    const std::vector<std::size_t>& sequence_lengths() const noexcept { return sequence_lengths_; }
    static constexpr PhysicalBlockID invalid_block() noexcept {
        return static_cast<PhysicalBlockID>(-1);
    }

    // out_of_range for an index outside the table or on a padding entry.
    PhysicalBlockID physical_id(std::size_t request, std::size_t logical_block) const;

private:
    friend BatchBlockTable build_batch_block_table(const std::vector<const SequenceState*>&);
    std::size_t max_blocks_per_sequence_ = 0;
    std::vector<PhysicalBlockID> block_table_;
    std::vector<std::size_t> sequence_lengths_;
};

BatchBlockTable build_batch_block_table(const std::vector<const SequenceState*>& sequences);

} // namespace kvflux::v2
