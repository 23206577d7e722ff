#pragma once
// Full-block prefix sharing on top of PhysicalBlockPool's publish/lookup
// (reference: include/kvflux/v2/prefix_cache.h:9-27). Metadata only.
#include "kvflux/v2/sequence_state.h"

namespace kvflux::v2 {

class PrefixCache {
public:
    explicit PrefixCache(PhysicalBlockPool& pool) noexcept : pool_(pool) {}

    // Attaches published full blocks matching the leading tokens to an empty
    // sequence, stopping at the first miss; returns the shared token count.
    // On an exception every block attached by this call is released.
    std::size_t attach_cached_prefix(SequenceState& sequence, const Tokens& tokens);

    // Publishes logical block `logical_block` of `sequence` under `prefix`
    // (all tokens from the start through the end of that block).
    void publish_computed_block(const SequenceState& sequence, std::size_t logical_block,
                                const Tokens& prefix);

private:
    PhysicalBlockPool& pool_;
};

} // namespace kvflux::v2
