// One sequence's page ids in logical order (reference: src/v2/paged_kv_read_table.cpp:5-12).
#include "kvflux/v2/paged_kv_read.h"

namespace kvflux::v2 {

ReadBlockTable build_read_block_table(const SequenceState& sequence) {
    ReadBlockTable ids;
    ids.reserve(sequence.num_allocated_blocks());
    for (std::size_t j = 0; j < sequence.num_allocated_blocks(); ++j) {
        ids.push_back(sequence.physical_block_id(j));
    }
    return ids;
}

} // namespace kvflux::v2
