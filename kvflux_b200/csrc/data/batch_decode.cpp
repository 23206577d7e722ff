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

namespace {

// Device address of page-locked host memory, or invalid_argument.
const void* pinned_address(const void* p, const char* name) {
    cudaPointerAttributes a{};
    const cudaError_t e = cudaPointerGetAttributes(&a, p);
    if (p == nullptr || e != cudaSuccess || a.type != cudaMemoryTypeHost || a.devicePointer == nullptr) {
        if (e != cudaSuccess) (void)cudaGetLastError();
        throw std::invalid_argument(std::string(name) + " must be page-locked host memory");
    }
    return a.devicePointer;
}

} // namespace

std::vector<TokenLocation> BatchDecodeSession::step_host(const void* key_host, const void* value_host,
                                                         const float* query_host, float* output_host) {
    if (failed_) throw std::logic_error("batch decode session failed earlier");
    const PagedKVLayout& layout = storage_.layout();
    const std::size_t batch = sequences_.size();
    const std::size_t kv_row = layout.num_kv_heads() * layout.head_size() * layout.element_bytes();
    const std::size_t q_row = query_heads_ * layout.head_size() * sizeof(float);
    const std::size_t kv_bytes = detail::mul_checked(batch, kv_row, "batch decode");
    const std::size_t q_bytes = detail::mul_checked(batch, q_row, "batch decode");

    detail::DeviceGuard guard(storage_.device());
    (void)pinned_address(key_host, "K");
    (void)pinned_address(value_host, "V");
    (void)pinned_address(query_host, "Q");
    auto* o_dev = static_cast<float*>(const_cast<void*>(pinned_address(output_host, "attention output")));
    if (detail::overlaps(output_host, q_bytes, query_host, q_bytes) ||
        detail::overlaps(output_host, q_bytes, key_host, kv_bytes) ||
        detail::overlaps(output_host, q_bytes, value_host, kv_bytes)) {
        throw std::invalid_argument("attention output must not overlap K, V or Q");
    }

    detail::StorageRuntime& rt = storage_.runtime();
    // Device staging for the step's inputs: K rows, V rows, Q rows.
    const std::size_t kv_al = (kv_bytes + 255) & ~std::size_t(255);
    auto* io = static_cast<unsigned char*>(rt.ensure_io(2 * kv_al + q_bytes));
    unsigned char* k_dev = io;
    unsigned char* v_dev = io + kv_al;
    auto* q_dev = reinterpret_cast<float*>(io + 2 * kv_al);
    // Rows go in two chunks: the first quarter's inputs go up and its launch
    // starts as soon as the pages are booked; the rest goes up on a side
    // stream meanwhile and runs there concurrently (as paged_attention_batch_host).
    const std::size_t head_rows = batch >= 16 ? (batch + 3) / 4 : batch;
    auto upload = [&](std::size_t r0, std::size_t r1, cudaStream_t st) {
        if (r1 <= r0) return;
        detail::cuda_check(cudaMemcpyAsync(k_dev + r0 * kv_row, static_cast<const unsigned char*>(key_host) + r0 * kv_row,
                                           (r1 - r0) * kv_row, cudaMemcpyHostToDevice, st), "upload K");
        detail::cuda_check(cudaMemcpyAsync(v_dev + r0 * kv_row,
                                           static_cast<const unsigned char*>(value_host) + r0 * kv_row,
                                           (r1 - r0) * kv_row, cudaMemcpyHostToDevice, st), "upload V");
        detail::cuda_check(cudaMemcpyAsync(reinterpret_cast<unsigned char*>(q_dev) + r0 * q_row,
                                           reinterpret_cast<const unsigned char*>(query_host) + r0 * q_row,
                                           (r1 - r0) * q_row, cudaMemcpyHostToDevice, st), "upload Q");
    };

    std::vector<TokenLocation> where;
    where.reserve(batch);
    try {
        upload(0, head_rows, nullptr);
        if (head_rows < batch) rt.ensure_side();
        std::vector<std::uint64_t> lens(batch), slots(batch);
        std::size_t total = 0, widest = 0;
        const std::size_t bs = layout.block_size();
        for (std::size_t r = 0; r < batch; ++r) {
            SequenceState& s = *sequences_[r];
            const TokenLocation loc = append_token_cow(storage_, s);
            where.push_back(loc);
            if (loc.physical_block >= layout.num_blocks()) throw std::out_of_range("batch decode block out of range");
            lens[r] = s.num_tokens();
            slots[r] = loc.physical_block * bs + loc.offset_in_block;
            total += lens[r];
            widest = std::max(widest, s.num_allocated_blocks());
        }
        if (widest > width_) allocate_table(widest + kHeadroomPages);

        const std::size_t bytes[2] = {batch * sizeof(std::uint64_t), batch * sizeof(std::uint64_t)};
        const void* host[2] = {lens.data(), slots.data()};
        void* dev[2] = {nullptr, nullptr};
        rt.upload(host, bytes, 2, dev);
        const auto* lens_d = static_cast<const uint64_t*>(dev[0]);
        const auto* slots_d = static_cast<const uint64_t*>(dev[1]);
        const uint32_t qh = static_cast<uint32_t>(query_heads_);
        const std::size_t max_len = *std::max_element(lens.begin(), lens.end());
        // One split size for all rows: each row is computed as by one launch.
        const uint32_t pps = kvfx_decode_pages_per_split(&rt.cache, batch, qh, max_len, total);
        auto chunk_max = [&](std::size_t r0, std::size_t r1) {
            return *std::max_element(lens.begin() + r0, lens.begin() + r1);
        };
        auto ws_of = [&](std::size_t r0, std::size_t r1) {
            const std::size_t b = kvfx_decode_workspace_bytes(&rt.cache, r1 - r0, qh, chunk_max(r0, r1), pps);
            return (b + 255) & ~std::size_t(255);
        };
        const std::size_t ws0 = ws_of(0, head_rows);
        const std::size_t ws1 = head_rows < batch ? ws_of(head_rows, batch) : 0;
        void* ws_head = rt.ensure_workspace(ws0, 0);
        void* ws_rest = rt.ensure_workspace(ws1, 1);
        auto launch = [&](std::size_t r0, std::size_t r1, void* w, std::size_t wb, cudaStream_t st) {
            detail::check_kvfx(
                kvfx_decode_append(&rt.cache, k_dev + r0 * kv_row, v_dev + r0 * kv_row, slots_d + r0,
                                   reinterpret_cast<const float*>(reinterpret_cast<const unsigned char*>(q_dev) +
                                                                  r0 * q_row),
                                   reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(o_dev) + r0 * q_row),
                                   table_ + r0 * width_, lens_d + r0, r1 - r0, width_, qh, chunk_max(r0, r1), pps, w,
                                   wb, st),
                "batch decode step");
        };
        if (head_rows < batch) {
            // The side stream starts after the lengths, slots and any page
            // copies issued on the default stream so far.
            detail::cuda_check(cudaEventRecord(rt.side_ready, nullptr), "record side start");
            detail::cuda_check(cudaStreamWaitEvent(rt.side, rt.side_ready, 0), "order side start");
        }
        launch(0, head_rows, ws_head, rt.workspace_size(0), nullptr);
        if (head_rows < batch) {
            upload(head_rows, batch, rt.side);
            launch(head_rows, batch, ws_rest, rt.workspace_size(1), rt.side);
            detail::cuda_check(cudaEventRecord(rt.side_done, rt.side), "record side work");
            detail::cuda_check(cudaStreamWaitEvent(nullptr, rt.side_done, 0), "order side work");
        }
        rt.finish("batch decode step synchronize");
    } catch (...) {
        failed_ = !where.empty();
        (void)cudaDeviceSynchronize();
        throw;
    }
    return where;
}

} // namespace kvflux::v2
