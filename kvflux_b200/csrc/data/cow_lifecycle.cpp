// append_token_cow and SequenceLifecycle.
//
// append_token_cow keeps the reference's contract (src/v2/copy_on_write.cpp:7-16):
// the sequence appends one position, copying a shared partial last page to a
// private one through PagedKVStorage::copy_block first.
//
// SequenceLifecycle keeps the reference's states, checks and exception types
// (src/v2/sequence_lifecycle.cpp:14-86: prefill once, then decode steps, any
// failure after pages were taken finishes the request and returns them), but
// not its call sequence. The reference runs each step as write_paged_kv and
// then paged_attention: two table uploads, two launches, two synchronisations.
// Here a step validates every argument both calls would check, uploads what
// it needs in one copy and synchronises once:
//   prefill: the slot of every prompt token and the page list go up together;
//            the paged write and the causal attention are enqueued back to
//            back on the default stream;
//   decode:  one kvfx_decode_append launch writes the new token's K/V rows
//            into the cache and attends over the sequence including them
//            (on 16-bit caches with head_size 64/128 and block 16 a single
//            kernel; other shapes take the row copy and the generic attention
//            kernel, still behind one synchronisation).
#include <cuda_runtime_api.h>

#include <stdexcept>
#include <vector>

#include "kvflux/v2/copy_on_write.h"
#include "kvflux/v2/paged_attention.h"
#include "kvflux/v2/paged_kv_read.h"
#include "kvflux/v2/paged_kv_write.h"
#include "kvflux/v2/sequence_lifecycle.h"
#include "runtime.h"

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

namespace {

// The pointer checks write_paged_kv and paged_attention make for `tokens`
// rows of K/V and of Q/O (device memory of the storage's GPU; Q and O apart
// from each other and from the cache).
void check_step_buffers(const PagedKVStorage& storage, std::size_t tokens, std::size_t query_heads,
                        const void* key, const void* value, const float* query, const float* output) {
    const PagedKVLayout& layout = storage.layout();
    detail::require_device_pointer(key, storage.device(), "K_new");
    detail::require_device_pointer(value, storage.device(), "V_new");
    const std::size_t qo_bytes = detail::mul_checked(
        detail::mul_checked(detail::mul_checked(tokens, query_heads, "sequence step"), layout.head_size(),
                            "sequence step"),
        sizeof(float), "sequence step");
    detail::require_device_pointer(query, storage.device(), "Q");
    detail::require_device_pointer(output, storage.device(), "attention output");
    if (detail::overlaps(query, qo_bytes, output, qo_bytes) ||
        detail::overlaps(query, qo_bytes, storage.key_base(), layout.total_bytes()) ||
        detail::overlaps(output, qo_bytes, storage.key_base(), layout.total_bytes())) {
        throw std::invalid_argument("Q and attention output must not overlap each other or KV cache");
    }
}

}  // namespace

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
        SequenceState& seq = *sequence_;
        seq.append_tokens(token_count);
        detail::DeviceGuard guard(storage_.device());
        check_step_buffers(storage_, token_count, query_heads_, key_device, value_device, query_device,
                           output_device);
        // The prompt's pages are this request's own fresh pages, so its slots
        // (page * block_size + offset, in token order) are distinct.
        const ReadBlockTable pages = build_read_block_table(seq);
        const std::size_t bs = seq.block_size();
        detail::StorageRuntime& rt = storage_.runtime();
        void* host[2] = {nullptr, nullptr};
        void* dev[2] = {nullptr, nullptr};
        const std::size_t bytes[2] = {detail::mul_checked(token_count, sizeof(PhysicalSlot), "prefill"),
                                      detail::mul_checked(pages.size(), sizeof(PhysicalBlockID), "prefill")};
        rt.stage(bytes, 2, host, dev);
        auto* slots = static_cast<PhysicalSlot*>(host[0]);
        for (std::size_t t = 0; t < token_count; ++t) slots[t] = pages[t / bs] * bs + t % bs;
        auto* ids = static_cast<PhysicalBlockID*>(host[1]);
        for (std::size_t j = 0; j < pages.size(); ++j) ids[j] = pages[j];
        rt.push();
        detail::check_kvfx(kvfx_write(&rt.cache, key_device, value_device, static_cast<const uint64_t*>(dev[0]),
                                      token_count, nullptr),
                           "paged KV write");
        const uint32_t qh = static_cast<uint32_t>(query_heads_);
        void* ws = rt.ensure_workspace(kvfx_attention_workspace_bytes(&rt.cache, token_count, token_count, qh));
        detail::check_kvfx(kvfx_attention(&rt.cache, query_device, output_device,
                                          static_cast<const uint64_t*>(dev[1]), token_count, token_count, qh, ws,
                                          rt.workspace_bytes, nullptr),
                           "paged attention");
        rt.finish("prefill synchronize");
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
        SequenceState& seq = *sequence_;
        detail::DeviceGuard guard(storage_.device());
        check_step_buffers(storage_, 1, query_heads_, key_device, value_device, query_device, output_device);
        const TokenLocation where = append_token_cow(storage_, seq);
        const std::size_t len = seq.num_tokens();
        const std::size_t width = seq.num_allocated_blocks();
        detail::StorageRuntime& rt = storage_.runtime();
        // Staging: [slot, length] then the page row.
        void* host[2] = {nullptr, nullptr};
        void* dev[2] = {nullptr, nullptr};
        const std::size_t bytes[2] = {2 * sizeof(uint64_t), width * sizeof(PhysicalBlockID)};
        rt.stage(bytes, 2, host, dev);
        auto* head = static_cast<uint64_t*>(host[0]);
        head[0] = where.physical_block * seq.block_size() + where.offset_in_block;
        head[1] = len;
        seq.copy_physical_block_ids(static_cast<PhysicalBlockID*>(host[1]));
        rt.push();
        const uint32_t qh = static_cast<uint32_t>(query_heads_);
        const auto* meta = static_cast<const uint64_t*>(dev[0]);
        void* ws = rt.ensure_workspace(kvfx_decode_workspace_bytes(&rt.cache, 1, qh, len, 0));
        detail::check_kvfx(kvfx_decode_append(&rt.cache, key_device, value_device, meta, query_device, output_device,
                                              static_cast<uint64_t*>(dev[1]), meta + 1, 1, width, qh, len, 0, ws,
                                              rt.workspace_bytes, nullptr),
                           "decode step");
        rt.finish("decode synchronize");
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

}  // namespace kvflux::v2
