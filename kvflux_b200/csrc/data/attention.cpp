// paged_attention and paged_attention_batch: the reference's host contract
// (src/v2/paged_attention.cu:193-313) in the same check order; the kernels
// are reached through kvfx_attention / kvfx_decode.
#include <algorithm>
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

void paged_attention_prefill_batch(const PagedKVStorage& storage, const std::vector<const SequenceState*>& sequences,
                                   const std::vector<const float*>& queries_device,
                                   const std::vector<float*>& outputs_device,
                                   const std::vector<std::size_t>& query_tokens, std::size_t query_heads) {
    const std::size_t n = sequences.size();
    if (queries_device.size() != n || outputs_device.size() != n || query_tokens.size() != n) {
        throw std::invalid_argument("prefill batch arrays differ in length");
    }
    const PagedKVLayout& layout = storage.layout();
    // Per sequence, paged_attention's checks in its order.
    std::vector<std::size_t> live;       // sequences with queries
    std::vector<std::size_t> io_bytes(n, 0);
    std::vector<ReadBlockTable> tables(n);
    std::size_t widest = 0;
    for (std::size_t i = 0; i < n; ++i) {
        const SequenceState* seq = sequences[i];
        if (seq == nullptr) throw std::invalid_argument("null sequence in prefill batch");
        if (!storage.uses_pool(seq->block_table())) {
            throw std::invalid_argument("sequence and KV storage must use one physical pool");
        }
        if (seq->block_size() != layout.block_size() || query_heads == 0 ||
            query_heads % layout.num_kv_heads() != 0 || query_tokens[i] > seq->num_tokens()) {
            throw std::invalid_argument("invalid paged attention shape");
        }
        const std::size_t elements = detail::mul_checked(
            detail::mul_checked(query_tokens[i], query_heads, "paged attention"), layout.head_size(),
            "paged attention");
        io_bytes[i] = detail::mul_checked(elements, sizeof(float), "paged attention");
        if (query_tokens[i] == 0) continue;
        if (queries_device[i] == nullptr || outputs_device[i] == nullptr) {
            throw std::invalid_argument("Q and attention output device pointers are required");
        }
        tables[i] = build_read_block_table(*seq);
        for (const PhysicalBlockID b : tables[i]) {
            if (b >= layout.num_blocks()) throw std::out_of_range("attention block out of range");
        }
        widest = std::max(widest, tables[i].size());
        live.push_back(i);
    }
    if (live.empty()) return;
    detail::DeviceGuard guard(storage.device());
    for (const std::size_t i : live) {
        detail::require_device_pointer(queries_device[i], storage.device(), "Q");
        detail::require_device_pointer(outputs_device[i], storage.device(), "attention output");
        if (detail::overlaps(queries_device[i], io_bytes[i], outputs_device[i], io_bytes[i]) ||
            detail::overlaps(queries_device[i], io_bytes[i], storage.key_base(), layout.total_bytes()) ||
            detail::overlaps(outputs_device[i], io_bytes[i], storage.key_base(), layout.total_bytes())) {
            throw std::invalid_argument("Q and attention output must not overlap each other or KV cache");
        }
    }
    // One launch runs the sequences concurrently: an output must not overlap
    // another sequence's Q or O (one call after another would define it).
    for (const std::size_t i : live) {
        for (const std::size_t j : live) {
            if (i == j) continue;
            if (detail::overlaps(outputs_device[i], io_bytes[i], outputs_device[j], io_bytes[j]) ||
                detail::overlaps(outputs_device[i], io_bytes[i], queries_device[j], io_bytes[j])) {
                throw std::invalid_argument("prefill batch outputs must not overlap other sequences' Q or O");
            }
        }
    }
    const std::size_t rows = live.size();
    const std::size_t table_bytes = detail::mul_checked(detail::mul_checked(rows, widest, "paged attention"),
                                                        sizeof(PhysicalBlockID), "paged attention");
    std::vector<PhysicalBlockID> table(rows * widest, BatchBlockTable::invalid_block());
    for (std::size_t r = 0; r < rows; ++r) {
        const ReadBlockTable& t = tables[live[r]];
        std::copy(t.begin(), t.end(), table.begin() + r * widest);
    }
    detail::StorageRuntime& rt = storage.runtime();
    const void* host[1] = {table.data()};
    void* dev[1] = {nullptr};
    rt.upload(host, &table_bytes, 1, dev);
    const uint32_t qh = static_cast<uint32_t>(query_heads);
    std::size_t ws_bytes = 0;
    for (const std::size_t i : live) {
        ws_bytes = std::max<std::size_t>(
            ws_bytes, kvfx_attention_workspace_bytes(&rt.cache, query_tokens[i], sequences[i]->num_tokens(), qh));
    }
    void* ws = rt.ensure_workspace(ws_bytes);
    const auto* table_dev = static_cast<const uint64_t*>(dev[0]);
    for (std::size_t r0 = 0; r0 < rows; r0 += KVFX_MAX_PREFILL_SEQS) {
        const std::size_t r1 = std::min<std::size_t>(rows, r0 + KVFX_MAX_PREFILL_SEQS);
        const float* q[KVFX_MAX_PREFILL_SEQS];
        float* o[KVFX_MAX_PREFILL_SEQS];
        uint64_t qt[KVFX_MAX_PREFILL_SEQS], kt[KVFX_MAX_PREFILL_SEQS];
        for (std::size_t r = r0; r < r1; ++r) {
            const std::size_t i = live[r];
            q[r - r0] = queries_device[i];
            o[r - r0] = outputs_device[i];
            qt[r - r0] = query_tokens[i];
            kt[r - r0] = sequences[i]->num_tokens();
        }
        detail::check_kvfx(kvfx_attention_batch(&rt.cache, static_cast<uint32_t>(r1 - r0), q, o,
                                                table_dev + r0 * widest, widest, qt, kt, qh, ws,
                                                rt.workspace_bytes, nullptr),
                           "paged attention prefill batch");
    }
    rt.finish("paged attention prefill batch synchronize");
}

namespace {

// Device address of page-locked host memory (cudaHostAlloc / cudaHostRegister),
// or invalid_argument for anything else.
void* pinned_device_address(const void* p, const char* name) {
    cudaPointerAttributes a{};
    const cudaError_t e = cudaPointerGetAttributes(&a, p);
    if (e != cudaSuccess || a.type != cudaMemoryTypeHost || a.devicePointer == nullptr) {
        if (e != cudaSuccess) (void)cudaGetLastError();
        throw std::invalid_argument(std::string(name) + " must be page-locked host memory");
    }
    return a.devicePointer;
}

// Shared body of paged_attention_batch (device Q/O) and
// paged_attention_batch_host (page-locked host Q/O).
void batch_decode(const PagedKVStorage& storage, const std::vector<const SequenceState*>& sequences,
                  const float* query_device, float* output_device, std::size_t query_heads, bool host_io) {
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
    (void)table_bytes;
    (void)lengths_bytes;

    auto check_pointers = [&] {
        const std::size_t elements = detail::mul_checked(
            detail::mul_checked(batch, query_heads, "batch attention"), layout.head_size(), "batch attention");
        const std::size_t tensor_bytes = detail::mul_checked(elements, sizeof(float), "batch attention");
        if (query_device == nullptr || output_device == nullptr) {
            throw std::invalid_argument("Q and attention output device pointers are required");
        }
        if (host_io) {
            (void)pinned_device_address(query_device, "Q");
            (void)pinned_device_address(output_device, "attention output");
            if (detail::overlaps(query_device, tensor_bytes, output_device, tensor_bytes)) {
                throw std::invalid_argument("Q and attention output must not overlap");
            }
            if (batch > 65535) throw std::invalid_argument("batch above 65535 sequences");
            return;
        }
        detail::require_device_pointer(query_device, storage.device(), "Q");
        detail::require_device_pointer(output_device, storage.device(), "attention output");
        if (detail::overlaps(query_device, tensor_bytes, output_device, tensor_bytes) ||
            detail::overlaps(query_device, tensor_bytes, storage.key_base(), layout.total_bytes()) ||
            detail::overlaps(output_device, tensor_bytes, storage.key_base(), layout.total_bytes())) {
            throw std::invalid_argument("Q and attention output must not overlap each other or KV cache");
        }
        if (batch > 65535) throw std::invalid_argument("batch above 65535 sequences");
    };
    // The reference raises table errors before pointer errors: with a bad
    // pointer, the whole table is built (and checked) before that is raised.
    bool pointers_ok = true;
    try {
        check_pointers();
    } catch (...) {
        pointers_ok = false;
    }
    if (!pointers_ok) {
        (void)build_batch_block_table(sequences);
        check_pointers();
    }

    // The page table stays on the device between calls; this uploads the
    // lengths and whatever entries changed (one copy, one patch launch).
    const detail::ResidentTable::View table = rt.batch_table.refresh(rt, sequences, lens, widest, layout.num_blocks());
    rt.last_table_upload = table.h2d_bytes;
    const std::size_t width = table.width;
    const std::size_t row_bytes = width * sizeof(PhysicalBlockID);

    const std::size_t max_len = *std::max_element(lens.begin(), lens.end());
    std::size_t total = 0;
    for (const std::size_t l : lens) total += l;
    const uint32_t qh = static_cast<uint32_t>(query_heads);
    // One split size for the whole batch, so that every row is computed
    // exactly as by one launch over all rows.
    const uint32_t pps = kvfx_decode_pages_per_split(&rt.cache, batch, qh, max_len, total);
    const std::size_t row_elems = query_heads * layout.head_size();
    auto chunk_max = [&](std::size_t r0, std::size_t r1) {
        return *std::max_element(lens.begin() + r0, lens.begin() + r1);
    };
    auto workspace_of = [&](std::size_t r0, std::size_t r1) {
        const std::size_t b = kvfx_decode_workspace_bytes(&rt.cache, r1 - r0, qh, chunk_max(r0, r1), pps);
        return (b + 255) & ~std::size_t(255);
    };
    // Host I/O: Q goes up per chunk into device scratch just ahead of that
    // chunk's kernel; the kernels write O straight into the page-locked
    // output (its device mapping), so neither copy waits for the other work.
    const float* q_dev = query_device;
    float* o_dev = output_device;
    if (host_io) {
        q_dev = static_cast<const float*>(rt.ensure_io(batch * row_elems * sizeof(float)));
        o_dev = static_cast<float*>(pinned_device_address(output_device, "attention output"));
    }
    auto upload_q = [&](std::size_t r0, std::size_t r1, cudaStream_t stream) {
        if (!host_io || r1 <= r0) return;
        detail::cuda_check(cudaMemcpyAsync(const_cast<float*>(q_dev) + r0 * row_elems, query_device + r0 * row_elems,
                                           (r1 - r0) * row_elems * sizeof(float), cudaMemcpyHostToDevice, stream),
                           "upload Q");
    };
    auto launch_rows = [&](std::size_t r0, std::size_t r1, void* ws, std::size_t ws_bytes, cudaStream_t stream) {
        detail::check_kvfx(
            kvfx_decode(&rt.cache, q_dev + r0 * row_elems, o_dev + r0 * row_elems,
                        reinterpret_cast<const uint64_t*>(reinterpret_cast<const unsigned char*>(table.table) +
                                                          r0 * row_bytes),
                        table.lens + r0, r1 - r0, width, qh, chunk_max(r0, r1), pps, ws, ws_bytes, stream),
            "paged attention batch");
    };

    // Device Q: one launch over every row. Host Q: two chunks, so that the
    // kernel over the first quarter of the rows starts once its Q is up
    // while the rest of Q goes up on a side stream, whose launch over the
    // other rows (own workspace, same split size) then runs concurrently
    // and fills the SMs the first kernel's last CTAs leave idle.
    const std::size_t head_rows = host_io && batch >= 16 ? (batch + 3) / 4 : batch;
    const std::size_t ws0 = workspace_of(0, head_rows);
    const std::size_t ws1 = head_rows < batch ? workspace_of(head_rows, batch) : 0;
    void* ws_head = rt.ensure_workspace(ws0, 0);
    void* ws_rest = rt.ensure_workspace(ws1, 1);
    upload_q(0, head_rows, nullptr);
    if (head_rows < batch) {
        // The side stream does not wait for the default stream by itself:
        // order it after the table patch and the caller's earlier work.
        rt.ensure_side();
        detail::cuda_check(cudaEventRecord(rt.side_ready, nullptr), "record side start");
        detail::cuda_check(cudaStreamWaitEvent(rt.side, rt.side_ready, 0), "order side start");
    }
    launch_rows(0, head_rows, ws_head, rt.workspace_size(0), nullptr);
    if (head_rows < batch) {
        upload_q(head_rows, batch, rt.side);
        launch_rows(head_rows, batch, ws_rest, rt.workspace_size(1), rt.side);
        detail::cuda_check(cudaEventRecord(rt.side_done, rt.side), "record side work");
        detail::cuda_check(cudaStreamWaitEvent(nullptr, rt.side_done, 0), "order side work");
    }
    rt.finish("paged attention batch synchronize");
}

} // namespace

void paged_attention_batch(const PagedKVStorage& storage, const std::vector<const SequenceState*>& sequences,
                           const float* query_device, float* output_device, std::size_t query_heads) {
    batch_decode(storage, sequences, query_device, output_device, query_heads, false);
}

void paged_attention_batch_host(const PagedKVStorage& storage, const std::vector<const SequenceState*>& sequences,
                                const float* query_host, float* output_host, std::size_t query_heads) {
    batch_decode(storage, sequences, query_host, output_host, query_heads, true);
}

std::size_t paged_attention_batch_table_upload_bytes(const PagedKVStorage& storage) {
    return storage.runtime().last_table_upload;
}

} // namespace kvflux::v2
