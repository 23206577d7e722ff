// Whole-block prefix sharing (reference: src/v2/prefix_cache.cpp:7-57).
#include "kvflux/v2/prefix_cache.h"

#include <stdexcept>

namespace kvflux::v2 {

std::size_t PrefixCache::attach_cached_prefix(SequenceState& sequence, const Tokens& tokens) {
    if (!sequence.block_table().uses_pool(pool_)) {
        throw std::invalid_argument("sequence and prefix cache must share one physical pool");
    }
    if (sequence.num_tokens() != 0) throw std::invalid_argument("prefix attach needs an empty sequence");
    const std::size_t bs = pool_.block_size();
    Tokens prefix;
    prefix.reserve(tokens.size());
    try {
        for (std::size_t start = 0; tokens.size() - start >= bs; start += bs) {
            prefix.insert(prefix.end(), tokens.begin() + static_cast<std::ptrdiff_t>(start),
                          tokens.begin() + static_cast<std::ptrdiff_t>(start + bs));
            PhysicalBlockHandle hit{};
            if (!pool_.lookup(prefix, hit)) break;
            // lookup's reference is temporary; the table takes its own.
            try {
                sequence.append_cached_full_block(hit);
            } catch (...) {
                pool_.free(hit);
                throw;
            }
            pool_.free(hit);
        }
    } catch (...) {
        while (sequence.num_tokens() != 0) sequence.drop_last_full_block();
        throw;
    }
    return sequence.num_tokens();
}

void PrefixCache::publish_computed_block(const SequenceState& sequence, std::size_t logical_block,
                                         const Tokens& prefix) {
    if (!sequence.block_table().uses_pool(pool_)) {
        throw std::invalid_argument("sequence and prefix cache must share one physical pool");
    }
    const std::size_t bs = pool_.block_size();
    if (logical_block >= sequence.num_allocated_blocks() || prefix.size() % bs != 0 ||
        prefix.size() / bs != logical_block + 1 || prefix.size() > sequence.num_tokens()) {
        throw std::invalid_argument("publish needs the exact whole-block token prefix");
    }
    pool_.publish(sequence.block_handle(logical_block), prefix);
}

} // namespace kvflux::v2
