#pragma once
// Synchronous single-request prefill -> decode -> finish driver over the v2
// data plane (reference: include/kvflux/v2/sequence_lifecycle.h:12-47).
#include "kvflux/v2/paged_kv_storage.h"

#include <cstddef>
#include <optional>

namespace kvflux::v2 {

class SequenceLifecycle {
public:
    SequenceLifecycle(RequestID request_id, PhysicalBlockPool& pool,
                      PagedKVStorage& storage, std::size_t query_heads);
    ~SequenceLifecycle() noexcept { finish(); }
    SequenceLifecycle(const SequenceLifecycle&) = delete;
    SequenceLifecycle& operator=(const SequenceLifecycle&) = delete;
    SequenceLifecycle(SequenceLifecycle&&) = delete;
    SequenceLifecycle& operator=(SequenceLifecycle&&) = delete;

    // K/V [token_count][kv_heads][head_size], Q/O [token_count][query_heads][head_size].
    void prefill(std::size_t token_count, const void* key_device, const void* value_device,
                 const float* query_device, float* output_device);
    TokenLocation decode(const void* key_device, const void* value_device,
                         const float* query_device, float* output_device);

    void finish() noexcept;
    bool finished() const noexcept { return !sequence_.has_value(); }
    const SequenceState& sequence() const;

private:
    void abort_after_failure() noexcept;

    PagedKVStorage& storage_;
    std::optional<SequenceState> sequence_;
    std::size_t query_heads_;
    bool prefilled_ = false;
};

} // namespace kvflux::v2
