// Slot ids in batch order (reference: src/v2/slot_mapping.cpp:8-32): slot =
// physical page * block_size + offset in the page, for every (sequence,
// token position) of the batch, with the reference's checks and exception
// types (null sequence or mixed pools: invalid_argument; position past the
// sequence: out_of_range; stale page handle: invalid_argument; slot beyond
// 64 bits: overflow_error), raised for the first offending write.
//
// Arrangement: batches are runs of positions of one sequence (a prefill
// writes every position of one sequence; a decode step one position of each),
// so the page of the previous write is remembered and a write into the same
// page of the same sequence reuses its checked id and slot base instead of
// repeating the generation-checked lookup per token. Nothing changes the
// pool during the call, so a page checked once stays valid for its run.
#include "kvflux/v2/slot_mapping.h"

#include <limits>
#include <stdexcept>

namespace kvflux::v2 {

SlotMapping build_slot_mapping(const std::vector<TokenWrite>& batch) {
    static_assert(sizeof(std::size_t) <= sizeof(PhysicalSlot), "size_t must fit in a slot id");
    constexpr PhysicalSlot kMax = std::numeric_limits<PhysicalSlot>::max();
    SlotMapping slots;
    slots.reserve(batch.size());
    if (batch.empty()) return slots;
    if (batch.front().sequence == nullptr) throw std::invalid_argument("null sequence in slot mapping");
    const BlockTable& first = batch.front().sequence->block_table();

    const SequenceState* run_seq = nullptr;  // the page remembered from the previous write
    std::size_t run_block = 0;
    PhysicalSlot run_base = 0;  // page * block_size of that page
    for (const TokenWrite& w : batch) {
        const SequenceState* s = w.sequence;
        if (s == nullptr) throw std::invalid_argument("null sequence in slot mapping");
        if (s != run_seq && !first.shares_pool_with(s->block_table())) {
            throw std::invalid_argument("slot mapping batch must share one physical pool");
        }
        if (w.token_position >= s->num_tokens()) throw std::out_of_range("token index beyond the sequence");
        const std::size_t bs = s->block_size();
        const std::size_t block = w.token_position / bs;
        const auto off = static_cast<PhysicalSlot>(w.token_position % bs);
        if (s != run_seq || block != run_block) {
            const auto page = static_cast<PhysicalSlot>(s->physical_block_id(block));  // generation-checked
            // The page's last slot must fit: page * bs + (bs - 1).
            if (page > (kMax - (bs - 1)) / bs) {
                if (page > (kMax - off) / bs) throw std::overflow_error("physical slot id would overflow");
                slots.push_back(page * bs + off);  // this offset fits; a later one of the page may not
                run_seq = nullptr;
                continue;
            }
            run_seq = s;
            run_block = block;
            run_base = page * bs;
        }
        slots.push_back(run_base + off);
    }
    return slots;
}

}  // namespace kvflux::v2
