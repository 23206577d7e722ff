#pragma once
// Batch-ordered physical slot ids: slot = physical_block * block_size + offset
// (reference: include/kvflux/v2/slot_mapping.h:12-23).
#include "kvflux/v2/sequence_state.h"

#include <cstddef>
#include <cstdint>
#include <vector>

namespace kvflux::v2 {

using PhysicalSlot = std::uint64_t;
using SlotMapping = std::vector<PhysicalSlot>;

struct TokenWrite {
    const SequenceState* sequence;  // borrowed for the duration of the call
    std::size_t token_position;     // must already be reserved
};

SlotMapping build_slot_mapping(const std::vector<TokenWrite>& batch);

} // namespace kvflux::v2
