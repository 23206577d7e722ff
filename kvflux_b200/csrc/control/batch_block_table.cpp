// Padded row-major batch page table (reference: src/v2/batch_block_table.cpp:8-48).
#include "kvflux/v2/batch_block_table.h"

#include <limits>
#include <stdexcept>

namespace kvflux::v2 {

PhysicalBlockID BatchBlockTable::physical_id(std::size_t request, std::size_t logical_block) const {
    if (request >= num_sequences() || logical_block >= max_blocks_per_sequence_) {
        throw std::out_of_range("batch block table index out of range");
    }
    const PhysicalBlockID id = block_table_[request * max_blocks_per_sequence_ + logical_block];
    if (id == invalid_block()) throw std::out_of_range("batch block table entry is padding");
    return id;
}

BatchBlockTable build_batch_block_table(const std::vector<const SequenceState*>& sequences) {
    BatchBlockTable out;
    if (sequences.empty()) return out;
    const SequenceState* first = sequences.front();
    if (first == nullptr) throw std::invalid_argument("null sequence in batch");

    out.sequence_lengths_.reserve(sequences.size());
    std::size_t widest = 0;
    for (const SequenceState* s : sequences) {
        if (s == nullptr) throw std::invalid_argument("null sequence in batch");
        if (!s->block_table().shares_pool_with(first->block_table())) {
            throw std::invalid_argument("batch sequences must share one physical pool");
        }
        out.sequence_lengths_.push_back(s->num_tokens());
        if (s->num_allocated_blocks() > widest) widest = s->num_allocated_blocks();
    }
    if (widest > std::numeric_limits<std::size_t>::max() / sequences.size()) {
        throw std::overflow_error("batch block table would overflow");
    }
    out.max_blocks_per_sequence_ = widest;
    out.block_table_.assign(sequences.size() * widest, BatchBlockTable::invalid_block());
    for (std::size_t r = 0; r < sequences.size(); ++r) {
        sequences[r]->copy_physical_block_ids(out.block_table_.data() + r * widest);
    }
    return out;
}

} // namespace kvflux::v2
