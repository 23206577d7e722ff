// One sequence's page ids in logical order (reference: src/v2/paged_kv_read_table.cpp:5-12).
#include "kvflux/v2/paged_kv_read.h"

namespace kvflux::v2 {

ReadBlockTable build_read_block_table(const SequenceState& sequence) {
    ReadBlockTable ids(sequence.num_allocated_blocks());
    sequence.copy_physical_block_ids(ids.data());
    return ids;
}

} // namespace kvflux::v2
