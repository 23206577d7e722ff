#pragma once
// Batched decode loop over the v2 data plane, with the padded 2-D block table
// resident on the device. The reference has no such class: it batches the
// decode step of SequenceLifecycle (src/v2/sequence_lifecycle.cpp:53-73:
// append with copy-on-write, slot mapping, paged KV write, attention of the
// last position) over many sequences, and replaces the per-call build and
// upload of the whole table (src/v2/batch_block_table.cpp:18-48,
// src/v2/paged_attention.cu:287-292) by the one entry per row that a step can
// change, written by the step's own launch (kvfx_decode_append).
#include "kvflux/v2/paged_kv_storage.h"
#include "kvflux/v2/sequence_state.h"

#include <cstddef>
#include <cstdint>
#include <vector>

namespace kvflux::v2 {

class BatchDecodeSession {
public:
    // `sequences`: distinct, non-null, non-empty (prefilled) sequences on the
    // storage's pool and block size; they must outlive the session. Between
    // steps they may change only through step(), or the caller re-reads them
    // with refresh(). query_heads: a positive multiple of the storage's KV
    // heads. Allocates the device table (its width leaves room for growth;
    // a step that outgrows it re-creates it).
    BatchDecodeSession(const PagedKVStorage& storage, std::vector<SequenceState*> sequences,
                       std::size_t query_heads);
    ~BatchDecodeSession() noexcept;
    BatchDecodeSession(const BatchDecodeSession&) = delete;
    BatchDecodeSession& operator=(const BatchDecodeSession&) = delete;

    // One decode step for every sequence, in batch order: appends one token
    // (copy-on-write of a shared partial last page, as append_token_cow), then
    // one launch writes key/value [batch][kv_heads][head_size] (device, the
    // storage's dtype) into the new slots and computes the attention of
    // query [batch][query_heads][head_size] (device float, the new position)
    // into output. Synchronous, like the reference's entry points. Returns
    // the new tokens' locations. If it throws after appending, the sequences
    // keep their new positions without K/V and the session refuses further
    // steps (logic_error): finish those requests, as SequenceLifecycle does.
    std::vector<TokenLocation> step(const void* key_device, const void* value_device,
                                    const float* query_device, float* output_device);

    // step() with key, value, query and output in page-locked host memory
    // (cudaHostAlloc / cudaHostRegister): the inputs go up in two row chunks,
    // each just ahead of its launch, and the launches write the output
    // straight into the host buffer, so the transfers overlap the attention.
    // Same results as step() on device copies of the same inputs.
    std::vector<TokenLocation> step_host(const void* key_host, const void* value_host,
                                         const float* query_host, float* output_host);

    // Re-reads row `row` (or every row) of the device table from its sequence.
    void refresh(std::size_t row);
    void refresh_all();

    std::size_t batch_size() const noexcept { return sequences_.size(); }
    std::size_t table_width() const noexcept { return width_; }
    // Device address of the row-major uint64 [batch][table_width()] table.
    const std::uint64_t* device_table() const noexcept { return table_; }

private:
    void allocate_table(std::size_t width);
    void upload_rows(std::size_t r0, std::size_t r1);

    const PagedKVStorage& storage_;
    std::vector<SequenceState*> sequences_;
    std::size_t query_heads_;
    std::size_t width_ = 0;
    std::uint64_t* table_ = nullptr;
    bool failed_ = false;
};

} // namespace kvflux::v2
