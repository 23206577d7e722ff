// paged_attention and paged_attention_batch: the reference's host contract
// (src/v2/paged_attention.cu:193-313) in the same check order; the kernels
// are reached through kvfx_attention / kvfx_decode.
#include <algorithm>
#include <atomic>
#include <cstring>
#include <limits>

#include "kvflux/v2/batch_block_table.h"
#include "kvflux/v2/paged_attention.h"
#include "kvflux/v2/paged_kv_read.h"
#include "runtime.h"

namespace kvflux::v2 {

void paged_attention(const PagedKVStorage& storage, const SequenceState& sequence, const float* query_device,
                     float* output_device, std::size_t query_tokens, std::size_t query_heads) {
    if (!storage.uses_pool(sequence.block_table())) {
        throw std::invalid_argument("sequence and KV storage must use one physical pool");
    }
    const PagedKVLayout& layout = storage.layout();
    if (sequence.block_size() != layout.block_size() || query_heads == 0 ||
        query_heads % layout.num_kv_heads() != 0 || query_tokens > sequence.num_tokens()) {
        throw std::invalid_argument("invalid paged attention shape");
    }
    const std::size_t elements = detail::mul_checked(
        detail::mul_checked(query_tokens, query_heads, "paged attention"), layout.head_size(), "paged attention");
    const std::size_t out_bytes = detail::mul_checked(elements, sizeof(float), "paged attention");
    if (query_tokens == 0) return;
    if (query_device == nullptr || output_device == nullptr) {
        throw std::invalid_argument("Q and attention output device pointers are required");
    }
    const ReadBlockTable blocks = build_read_block_table(sequence);
    for (const PhysicalBlockID b : blocks) {
        if (b >= layout.num_blocks()) throw std::out_of_range("attention block out of range");
    }
    const std::size_t table_bytes = detail::mul_checked(blocks.size(), sizeof(PhysicalBlockID), "paged attention");

    detail::DeviceGuard guard(storage.device());
    detail::require_device_pointer(query_device, storage.device(), "Q");
    detail::require_device_pointer(output_device, storage.device(), "attention output");
    if (detail::overlaps(query_device, out_bytes, output_device, out_bytes) ||
        detail::overlaps(query_device, out_bytes, storage.key_base(), layout.total_bytes()) ||
        detail::overlaps(output_device, out_bytes, storage.key_base(), layout.total_bytes())) {
        throw std::invalid_argument("Q and attention output must not overlap each other or KV cache");
    }
    detail::StorageRuntime& rt = storage.runtime();
    const void* host[1] = {blocks.data()};
    void* dev[1] = {nullptr};
    rt.upload(host, &table_bytes, 1, dev);
    const uint32_t qh = static_cast<uint32_t>(query_heads);
    const std::size_t ws_bytes =
        kvfx_attention_workspace_bytes(&rt.cache, query_tokens, sequence.num_tokens(), qh);
    void* ws = rt.ensure_workspace(ws_bytes);
    detail::check_kvfx(kvfx_attention(&rt.cache, query_device, output_device,
                                      static_cast<const uint64_t*>(dev[0]), query_tokens,
                                      sequence.num_tokens(), qh, ws, rt.workspace_bytes, nullptr),
                       "paged attention");
    rt.finish("paged attention synchronize");
}

void paged_attention_batch(const PagedKVStorage& storage, const std::vector<const SequenceState*>& sequences,
                           const float* query_device, float* output_device, std::size_t query_heads) {
    const PagedKVLayout& layout = storage.layout();
    if (query_heads == 0 || query_heads % layout.num_kv_heads() != 0) {
        throw std::invalid_argument("invalid batch attention head count");
    }
    if (sequences.empty()) return;
    // The checks of build_batch_block_table and of the batch, in the same
    // order; the padded table itself is written straight into the pinned
    // staging below instead of a host vector that is then copied.
    const SequenceState* first = sequences.front();
    if (first == nullptr) throw std::invalid_argument("null sequence in batch");
    const std::size_t batch = sequences.size();
    std::vector<std::size_t> lens(batch);
    std::size_t widest = 0;
    for (std::size_t r = 0; r < batch; ++r) {
        const SequenceState* s = sequences[r];
        if (s == nullptr) throw std::invalid_argument("null sequence in batch");
        if (!s->block_table().shares_pool_with(first->block_table())) {
            throw std::invalid_argument("batch sequences must share one physical pool");
        }
        lens[r] = s->num_tokens();
        widest = std::max(widest, s->num_allocated_blocks());
    }
    if (widest > std::numeric_limits<std::size_t>::max() / batch) {
        throw std::overflow_error("batch block table would overflow");
    }
    for (std::size_t r = 0; r < batch; ++r) {
        if (!storage.uses_pool(sequences[r]->block_table()) || sequences[r]->block_size() != layout.block_size() ||
            lens[r] == 0) {
            throw std::invalid_argument("invalid batch attention sequence");
        }
    }
    const std::size_t table_bytes = detail::mul_checked(batch * widest, sizeof(PhysicalBlockID), "batch attention");
    const std::size_t lengths_bytes = detail::mul_checked(batch, sizeof(std::size_t), "batch attention");

    detail::DeviceGuard guard(storage.device());
    detail::StorageRuntime& rt = storage.runtime();
    void* host[2] = {nullptr, nullptr};
    void* dev[2] = {nullptr, nullptr};
    const std::size_t bytes[2] = {table_bytes, lengths_bytes};
    rt.stage(bytes, 2, host, dev);
    // Rows are independent: filled in parallel, page ids range-checked as
    // they are written. Any exception from the control plane is reproduced
    // by the sequential build, so that the first failing row raises it.
    auto* table = static_cast<PhysicalBlockID*>(host[0]);
    const std::size_t num_blocks = layout.num_blocks();
    std::atomic<bool> bad{false};
    try {
        detail::parallel_for(batch, 8, [&](std::size_t r0, std::size_t r1) {
            bool out_of_range = false;
            for (std::size_t r = r0; r < r1; ++r) {
                PhysicalBlockID* row = table + r * widest;
                const SequenceState& s = *sequences[r];
                const std::size_t n = s.num_allocated_blocks();
                for (std::size_t j = 0; j < n; ++j) {
                    const PhysicalBlockID id = s.physical_block_id(j);
                    out_of_range |= id >= num_blocks;
                    row[j] = id;
                }
                std::fill(row + n, row + widest, BatchBlockTable::invalid_block());
            }
            if (out_of_range) bad.store(true, std::memory_order_relaxed);
        });
    } catch (...) {
        (void)build_batch_block_table(sequences);
        throw;
    }
    if (bad.load()) throw std::out_of_range("batch attention block out of range");

    const std::size_t elements = detail::mul_checked(
        detail::mul_checked(batch, query_heads, "batch attention"), layout.head_size(), "batch attention");
    const std::size_t tensor_bytes = detail::mul_checked(elements, sizeof(float), "batch attention");
    if (query_device == nullptr || output_device == nullptr) {
        throw std::invalid_argument("Q and attention output device pointers are required");
    }
    detail::require_device_pointer(query_device, storage.device(), "Q");
    detail::require_device_pointer(output_device, storage.device(), "attention output");
    if (detail::overlaps(query_device, tensor_bytes, output_device, tensor_bytes) ||
        detail::overlaps(query_device, tensor_bytes, storage.key_base(), layout.total_bytes()) ||
        detail::overlaps(output_device, tensor_bytes, storage.key_base(), layout.total_bytes())) {
        throw std::invalid_argument("Q and attention output must not overlap each other or KV cache");
    }
    if (batch > 65535) throw std::invalid_argument("batch above 65535 sequences");

    std::memcpy(host[1], lens.data(), lengths_bytes);
    const std::size_t max_len = *std::max_element(lens.begin(), lens.end());
    std::size_t total = 0;
    for (const std::size_t l : lens) total += l;
    rt.push();
    const uint32_t qh = static_cast<uint32_t>(query_heads);
    const uint32_t pps = kvfx_decode_pages_per_split(&rt.cache, batch, qh, max_len, total);
    const std::size_t ws_bytes = kvfx_decode_workspace_bytes(&rt.cache, batch, qh, max_len, pps);
    void* ws = rt.ensure_workspace(ws_bytes);
    detail::check_kvfx(kvfx_decode(&rt.cache, query_device, output_device, static_cast<const uint64_t*>(dev[0]),
                                   static_cast<const uint64_t*>(dev[1]), batch, widest, qh, max_len, pps, ws,
                                   rt.workspace_bytes, nullptr),
                       "paged attention batch");
    rt.finish("paged attention batch synchronize");
}

} // namespace kvflux::v2
