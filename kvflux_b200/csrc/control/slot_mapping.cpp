// Slot ids in batch order (reference: src/v2/slot_mapping.cpp:8-32).
#include "kvflux/v2/slot_mapping.h"

#include <limits>
#include <stdexcept>

namespace kvflux::v2 {

SlotMapping build_slot_mapping(const std::vector<TokenWrite>& batch) {
    static_assert(sizeof(std::size_t) <= sizeof(PhysicalSlot), "size_t must fit in a slot id");
    SlotMapping slots;
    slots.reserve(batch.size());
    if (batch.empty()) return slots;
    if (batch.front().sequence == nullptr) throw std::invalid_argument("null sequence in slot mapping");
    const BlockTable& first = batch.front().sequence->block_table();
    for (const TokenWrite& w : batch) {
        if (w.sequence == nullptr) throw std::invalid_argument("null sequence in slot mapping");
        if (!first.shares_pool_with(w.sequence->block_table())) {
            throw std::invalid_argument("slot mapping batch must share one physical pool");
        }
        const TokenLocation loc = w.sequence->token_location(w.token_position);
        const auto bs = static_cast<PhysicalSlot>(w.sequence->block_size());
        const auto page = static_cast<PhysicalSlot>(loc.physical_block);
        const auto off = static_cast<PhysicalSlot>(loc.offset_in_block);
        if (page > (std::numeric_limits<PhysicalSlot>::max() - off) / bs) {
            throw std::overflow_error("physical slot id would overflow");
        }
        slots.push_back(page * bs + off);
    }
    return slots;
}

} // namespace kvflux::v2
