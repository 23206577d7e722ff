#pragma once
// Gather of one sequence's pages into contiguous device K/V
// [num_tokens][num_kv_heads][head_size] (reference:
// include/kvflux/v2/paged_kv_read.h:10-19). Synchronous on the legacy default
// stream; an empty sequence returns before touching the output pointers.
#include "kvflux/v2/paged_kv_storage.h"

#include <vector>

namespace kvflux::v2 {

using ReadBlockTable = std::vector<PhysicalBlockID>;
ReadBlockTable build_read_block_table(const SequenceState& sequence);

void read_paged_kv(const PagedKVStorage& storage, const SequenceState& sequence,
                   void* key_out_device, void* value_out_device);

} // namespace kvflux::v2
