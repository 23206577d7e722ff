// append_token_cow and SequenceLifecycle (reference: src/v2/copy_on_write.cpp:7-16,
// src/v2/sequence_lifecycle.cpp:14-86).
#include <cuda_runtime_api.h>

#include "kvflux/v2/copy_on_write.h"
#include "kvflux/v2/paged_attention.h"
#include "kvflux/v2/paged_kv_write.h"
#include "kvflux/v2/sequence_lifecycle.h"

#include <stdexcept>
#include <vector>

namespace kvflux::v2 {

TokenLocation append_token_cow(const PagedKVStorage& storage, SequenceState& sequence) {
    if (!storage.uses_pool(sequence.block_table()) || storage.layout().block_size() != sequence.block_size()) {
        throw std::invalid_argument("sequence and KV storage must use one physical pool");
    }
    return sequence.append_token_with_copy(
        [&](PhysicalBlockHandle source, PhysicalBlockHandle destination) {
            storage.copy_block(source, destination);
        });
}

SequenceLifecycle::SequenceLifecycle(RequestID request_id, PhysicalBlockPool& pool, PagedKVStorage& storage,
                                     std::size_t query_heads)
    : storage_(storage), sequence_(std::in_place, request_id, pool), query_heads_(query_heads) {
    if (!storage_.uses_pool(sequence_->block_table()) || query_heads_ == 0 ||
        query_heads_ % storage_.layout().num_kv_heads() != 0) {
        throw std::invalid_argument("invalid sequence lifecycle pool or query head count");
    }
}

const SequenceState& SequenceLifecycle::sequence() const {
    if (finished()) throw std::logic_error("request has finished");
    return *sequence_;
}

void SequenceLifecycle::prefill(std::size_t token_count, const void* key_device, const void* value_device,
                                const float* query_device, float* output_device) {
    if (finished() || prefilled_) throw std::logic_error("request cannot prefill again");
    if (token_count == 0 || !key_device || !value_device || !query_device || !output_device) {
        throw std::invalid_argument("prefill requires tokens and device buffers");
    }
    try {
        sequence_->append_tokens(token_count);
        std::vector<TokenWrite> writes;
        writes.reserve(token_count);
        for (std::size_t t = 0; t < token_count; ++t) writes.push_back({&*sequence_, t});
        write_paged_kv(storage_, key_device, value_device, build_slot_mapping(writes));
        paged_attention(storage_, *sequence_, query_device, output_device, token_count, query_heads_);
        prefilled_ = true;
    } catch (...) {
        abort_after_failure();
        throw;
    }
}

TokenLocation SequenceLifecycle::decode(const void* key_device, const void* value_device,
                                        const float* query_device, float* output_device) {
    if (finished() || !prefilled_) throw std::logic_error("request must prefill before decode");
    if (!key_device || !value_device || !query_device || !output_device) {
        throw std::invalid_argument("decode requires device buffers");
    }
    try {
        const std::size_t position = sequence_->num_tokens();
        const TokenLocation where = append_token_cow(storage_, *sequence_);
        write_paged_kv(storage_, key_device, value_device, build_slot_mapping({{&*sequence_, position}}));
        paged_attention(storage_, *sequence_, query_device, output_device, 1, query_heads_);
        return where;
    } catch (...) {
        abort_after_failure();
        throw;
    }
}

void SequenceLifecycle::finish() noexcept {
    sequence_.reset();
    prefilled_ = false;
}

void SequenceLifecycle::abort_after_failure() noexcept {
    int previous = 0;
    if (cudaGetDevice(&previous) == cudaSuccess && cudaSetDevice(storage_.device()) == cudaSuccess) {
        (void)cudaDeviceSynchronize();  // no kernel may still touch pages about to be freed
        (void)cudaSetDevice(previous);
    }
    finish();
}

} // namespace kvflux::v2
