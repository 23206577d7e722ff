// BatchDecodeSession: batched decode steps with a device-resident block table
// (include/kvflux/v2/batch_decode_session.h). Each step is host page
// bookkeeping (append_token_cow per row), one small upload (new lengths and
// slots, 16 bytes per row) and one kvfx_decode_append launch.
#include "kvflux/v2/batch_decode_session.h"

#include <algorithm>
#include <cstring>
#include <limits>
#include <stdexcept>
#include <unordered_set>

#include "kvflux/v2/batch_block_table.h"
#include "kvflux/v2/copy_on_write.h"
#include "runtime.h"

namespace kvflux::v2 {

namespace {

// Columns of headroom beyond the widest row: 64 pages, 1024 tokens at block 16.
constexpr std::size_t kHeadroomPages = 64;

} // namespace

BatchDecodeSession::BatchDecodeSession(const PagedKVStorage& storage, std::vector<SequenceState*> sequences,
                                       std::size_t query_heads)
    : storage_(storage), sequences_(std::move(sequences)), query_heads_(query_heads) {
    const PagedKVLayout& layout = storage_.layout();
    if (query_heads_ == 0 || query_heads_ % layout.num_kv_heads() != 0) {
        throw std::invalid_argument("invalid batch decode head count");
    }
    if (sequences_.empty()) throw std::invalid_argument("batch decode needs at least one sequence");
    if (sequences_.size() > 65535) throw std::invalid_argument("batch above 65535 sequences");
    std::unordered_set<const SequenceState*> seen;
    std::size_t widest = 0;
    for (SequenceState* s : sequences_) {
        if (s == nullptr) throw std::invalid_argument("null sequence in batch");
        if (!seen.insert(s).second) throw std::invalid_argument("a sequence appears twice in the batch");
        if (!storage_.uses_pool(s->block_table()) || s->block_size() != layout.block_size() ||
            s->num_tokens() == 0) {
            throw std::invalid_argument("invalid batch decode sequence");
        }
        widest = std::max(widest, s->num_allocated_blocks());
    }
    detail::DeviceGuard guard(storage_.device());
    allocate_table(widest + kHeadroomPages);
}

BatchDecodeSession::~BatchDecodeSession() noexcept {
    if (table_ != nullptr) {
        int previous = 0;
        if (cudaGetDevice(&previous) == cudaSuccess && cudaSetDevice(storage_.device()) == cudaSuccess) {
            (void)cudaFree(table_);
            (void)cudaSetDevice(previous);
        }
    }
}

void BatchDecodeSession::allocate_table(std::size_t width) {
    const std::size_t batch = sequences_.size();
    if (width > std::numeric_limits<std::size_t>::max() / batch / sizeof(std::uint64_t)) {
        throw std::overflow_error("batch decode table would overflow");
    }
    void* fresh = nullptr;
    detail::cuda_check(cudaMalloc(&fresh, batch * width * sizeof(std::uint64_t)), "allocate batch decode table");
    if (table_ != nullptr) (void)cudaFree(table_);
    table_ = static_cast<std::uint64_t*>(fresh);
    width_ = width;
    upload_rows(0, batch);
}

void BatchDecodeSession::upload_rows(std::size_t r0, std::size_t r1) {
    if (r0 >= r1) return;
    const std::size_t num_blocks = storage_.layout().num_blocks();
    std::vector<PhysicalBlockID> rows((r1 - r0) * width_, BatchBlockTable::invalid_block());
    for (std::size_t r = r0; r < r1; ++r) {
        const SequenceState& s = *sequences_[r];
        if (s.num_allocated_blocks() > width_) throw std::logic_error("batch decode row outgrew its table");
        PhysicalBlockID* row = rows.data() + (r - r0) * width_;
        s.copy_physical_block_ids(row);
        for (std::size_t j = 0; j < s.num_allocated_blocks(); ++j) {
            if (row[j] >= num_blocks) throw std::out_of_range("batch decode block out of range");
        }
    }
    detail::cuda_check(cudaMemcpy(table_ + r0 * width_, rows.data(), rows.size() * sizeof(PhysicalBlockID),
                                  cudaMemcpyHostToDevice),
                       "upload batch decode table");
}

void BatchDecodeSession::refresh(std::size_t row) {
    if (row >= sequences_.size()) throw std::out_of_range("batch decode row out of range");
    detail::DeviceGuard guard(storage_.device());
    const std::size_t need = sequences_[row]->num_allocated_blocks();
    if (need > width_) {
        allocate_table(need + kHeadroomPages);  // re-reads every row
    } else {
        upload_rows(row, row + 1);
    }
}

void BatchDecodeSession::refresh_all() {
    detail::DeviceGuard guard(storage_.device());
    std::size_t widest = 0;
    for (const SequenceState* s : sequences_) widest = std::max(widest, s->num_allocated_blocks());
    if (widest > width_) {
        allocate_table(widest + kHeadroomPages);
    } else {
        upload_rows(0, sequences_.size());
    }
}

std::vector<TokenLocation> BatchDecodeSession::step(const void* key_device, const void* value_device,
                                                    const float* query_device, float* output_device) {
    if (failed_) throw std::logic_error("batch decode session failed earlier");
    const PagedKVLayout& layout = storage_.layout();
    const std::size_t batch = sequences_.size();
    if (key_device == nullptr || value_device == nullptr || query_device == nullptr || output_device == nullptr) {
        throw std::invalid_argument("batch decode requires device buffers");
    }
    const std::size_t kv_bytes = detail::mul_checked(
        detail::mul_checked(batch, layout.num_kv_heads() * layout.head_size(), "batch decode"),
        layout.element_bytes(), "batch decode");
    const std::size_t q_bytes = detail::mul_checked(
        detail::mul_checked(batch, query_heads_ * layout.head_size(), "batch decode"), sizeof(float),
        "batch decode");

    detail::DeviceGuard guard(storage_.device());
    detail::require_device_pointer(key_device, storage_.device(), "K");
    detail::require_device_pointer(value_device, storage_.device(), "V");
    detail::require_device_pointer(query_device, storage_.device(), "Q");
    detail::require_device_pointer(output_device, storage_.device(), "attention output");
    const void* cache = storage_.key_base();
    const std::size_t cache_bytes = layout.total_bytes();
    if (detail::overlaps(key_device, kv_bytes, cache, cache_bytes) ||
        detail::overlaps(value_device, kv_bytes, cache, cache_bytes) ||
        detail::overlaps(output_device, q_bytes, cache, cache_bytes) ||
        detail::overlaps(query_device, q_bytes, cache, cache_bytes) ||
        detail::overlaps(output_device, q_bytes, query_device, q_bytes) ||
        detail::overlaps(output_device, q_bytes, key_device, kv_bytes) ||
        detail::overlaps(output_device, q_bytes, value_device, kv_bytes)) {
        throw std::invalid_argument("K, V, Q and attention output must not overlap the KV cache or the output");
    }

    detail::StorageRuntime& rt = storage_.runtime();
    std::vector<TokenLocation> where;
    where.reserve(batch);
    try {
        std::vector<std::uint64_t> lens(batch), slots(batch);
        std::size_t max_len = 0, total = 0, widest = 0;
        const std::size_t bs = layout.block_size();
        for (std::size_t r = 0; r < batch; ++r) {
            SequenceState& s = *sequences_[r];
            const TokenLocation loc = append_token_cow(storage_, s);
            where.push_back(loc);
            if (loc.physical_block >= layout.num_blocks()) throw std::out_of_range("batch decode block out of range");
            lens[r] = s.num_tokens();
            slots[r] = loc.physical_block * bs + loc.offset_in_block;
            max_len = std::max<std::size_t>(max_len, lens[r]);
            total += lens[r];
            widest = std::max(widest, s.num_allocated_blocks());
        }
        if (widest > width_) allocate_table(widest + kHeadroomPages);

        const std::size_t bytes[2] = {batch * sizeof(std::uint64_t), batch * sizeof(std::uint64_t)};
        const void* host[2] = {lens.data(), slots.data()};
        void* dev[2] = {nullptr, nullptr};
        rt.upload(host, bytes, 2, dev);
        const uint32_t qh = static_cast<uint32_t>(query_heads_);
        const uint32_t pps = kvfx_decode_pages_per_split(&rt.cache, batch, qh, max_len, total);
        const std::size_t ws_bytes = kvfx_decode_workspace_bytes(&rt.cache, batch, qh, max_len, pps);
        void* ws = rt.ensure_workspace(ws_bytes);
        detail::check_kvfx(kvfx_decode_append(&rt.cache, key_device, value_device,
                                              static_cast<const uint64_t*>(dev[1]), query_device, output_device,
                                              table_, static_cast<const uint64_t*>(dev[0]), batch, width_, qh,
                                              max_len, pps, ws, rt.workspace_bytes, nullptr),
                           "batch decode step");
        rt.finish("batch decode step synchronize");
    } catch (...) {
        // A failure before the first append changed nothing (append_token_cow
        // is all-or-nothing per sequence); after it, the batch is inconsistent.
        failed_ = !where.empty();
        (void)cudaDeviceSynchronize();
        throw;
    }
    return where;
}

} // namespace kvflux::v2
