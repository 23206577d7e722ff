// paged_attention and paged_attention_batch: the reference's host contract
// (src/v2/paged_attention.cu:193-313) in the same check order; the kernels
// are reached through kvfx_attention / kvfx_decode.
#include <algorithm>

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
    const BatchBlockTable table = build_batch_block_table(sequences);
    for (std::size_t r = 0; r < sequences.size(); ++r) {
        if (!storage.uses_pool(sequences[r]->block_table()) || sequences[r]->block_size() != layout.block_size() ||
            table.sequence_lengths()[r] == 0) {
            throw std::invalid_argument("invalid batch attention sequence");
        }
    }
    for (const PhysicalBlockID b : table.block_table()) {
        if (b != BatchBlockTable::invalid_block() && b >= layout.num_blocks()) {
            throw std::out_of_range("batch attention block out of range");
        }
    }
    const std::size_t elements = detail::mul_checked(
        detail::mul_checked(sequences.size(), query_heads, "batch attention"), layout.head_size(), "batch attention");
    const std::size_t tensor_bytes = detail::mul_checked(elements, sizeof(float), "batch attention");
    if (sequences.empty()) return;
    if (query_device == nullptr || output_device == nullptr) {
        throw std::invalid_argument("Q and attention output device pointers are required");
    }
    const std::size_t table_bytes =
        detail::mul_checked(table.block_table().size(), sizeof(PhysicalBlockID), "batch attention");
    const std::size_t lengths_bytes = detail::mul_checked(sequences.size(), sizeof(std::size_t), "batch attention");

    detail::DeviceGuard guard(storage.device());
    detail::require_device_pointer(query_device, storage.device(), "Q");
    detail::require_device_pointer(output_device, storage.device(), "attention output");
    if (detail::overlaps(query_device, tensor_bytes, output_device, tensor_bytes) ||
        detail::overlaps(query_device, tensor_bytes, storage.key_base(), layout.total_bytes()) ||
        detail::overlaps(output_device, tensor_bytes, storage.key_base(), layout.total_bytes())) {
        throw std::invalid_argument("Q and attention output must not overlap each other or KV cache");
    }
    if (sequences.size() > 65535) throw std::invalid_argument("batch above 65535 sequences");

    detail::StorageRuntime& rt = storage.runtime();
    const std::vector<std::size_t>& lens = table.sequence_lengths();
    const std::size_t max_len = *std::max_element(lens.begin(), lens.end());
    std::size_t total = 0;
    for (const std::size_t l : lens) total += l;
    const void* host[2] = {table.block_table().data(), lens.data()};
    const std::size_t bytes[2] = {table_bytes, lengths_bytes};
    void* dev[2] = {nullptr, nullptr};
    rt.upload(host, bytes, 2, dev);
    const uint32_t qh = static_cast<uint32_t>(query_heads);
    const uint32_t pps = kvfx_decode_pages_per_split(&rt.cache, sequences.size(), qh, max_len, total);
    const std::size_t ws_bytes = kvfx_decode_workspace_bytes(&rt.cache, sequences.size(), qh, max_len, pps);
    void* ws = rt.ensure_workspace(ws_bytes);
    detail::check_kvfx(kvfx_decode(&rt.cache, query_device, output_device, static_cast<const uint64_t*>(dev[0]),
                                   static_cast<const uint64_t*>(dev[1]), sequences.size(),
                                   table.max_blocks_per_sequence(), qh, max_len, pps, ws,
                                   rt.workspace_bytes, nullptr),
                       "paged attention batch");
    rt.finish("paged attention batch synchronize");
}

} // namespace kvflux::v2
