#pragma once
// PagedAttention straight from the paged cache (reference:
// include/kvflux/v2/paged_attention.h:20-33). Q and O are FP32 device arrays;
// K/V are read in the storage dtype. Q heads are grouped onto KV heads
// (query_heads / num_kv_heads adjacent Q heads per KV head).
//
// paged_attention: one sequence, Q/O [query_tokens][query_heads][head_size],
//   Q aligned to the end of the sequence (query i sees positions
//   <= num_tokens - query_tokens + i): query_tokens == num_tokens is a causal
//   prefill, query_tokens == 1 a decode step.
// paged_attention_batch: one last-position query per sequence,
//   Q/O [num_sequences][query_heads][head_size].
// Both are synchronous on the legacy default stream and validate shapes,
// pointers and overlaps before launching.
//
// paged_attention_batch keeps the padded page table on the GPU between calls
// (per storage): a call uploads the sequence lengths and only the table
// entries that changed since the previous call (new pages, copied-on-write
// pages, rows of sequences not in the previous batch) instead of the whole
// table the reference uploads every call (src/v2/paged_attention.cu:287-292).
// Stale or foreign handles still raise what build_batch_block_table raises.
#include "kvflux/v2/paged_kv_storage.h"

#include <cstddef>
#include <vector>

namespace kvflux::v2 {

void paged_attention(const PagedKVStorage& storage, const SequenceState& sequence,
                     const float* query_device, float* output_device,
                     std::size_t query_tokens, std::size_t query_heads);

void paged_attention_batch(const PagedKVStorage& storage,
                           const std::vector<const SequenceState*>& sequences,
                           const float* query_device, float* output_device,
                           std::size_t query_heads);

// paged_attention_batch with Q and O in page-locked host memory
// (cudaHostAlloc / cudaHostRegister) instead of device memory; no
// counterpart in the reference, whose batch API takes device buffers. Same
// checks, results (bit-identical) and synchronous contract. Q goes up in row
// chunks, each just ahead of its kernel, and the kernels write O straight
// into the host buffer through its device mapping, so the transfers overlap
// the attention instead of preceding and following it.
void paged_attention_batch_host(const PagedKVStorage& storage,
                                const std::vector<const SequenceState*>& sequences,
                                const float* query_host, float* output_host,
                                std::size_t query_heads);

// Host->device bytes of tables and lengths the last paged_attention_batch(_host)
// call on `storage` uploaded (Q of the _host form not included). No
// counterpart in the reference.
std::size_t paged_attention_batch_table_upload_bytes(const PagedKVStorage& storage);

// paged_attention over several sequences of one storage in one call (a
// prefill batch); no counterpart in the reference, whose callers make one
// paged_attention call per sequence. Sequence i has query_tokens[i] queries
// in queries_device[i] and its output in outputs_device[i] (each
// [query_tokens[i]][query_heads][head_size] FP32 on the storage's device).
// paged_attention's checks run over the batch in two passes, each in
// sequence order: pool, shape, size overflow, null pointers and page ids of
// every sequence, then the device and overlap checks of every sequence; last,
// no output may overlap another sequence's Q or O (invalid_argument). The
// arrays must all have sequences.size() entries. Sequences with no queries
// are skipped. Outputs are bit-identical to one paged_attention per sequence; the
// tensor-core shapes of up to KVFX_MAX_PREFILL_SEQS sequences at a time share
// one persistent launch. Synchronous on the legacy default stream.
void paged_attention_prefill_batch(const PagedKVStorage& storage,
                                   const std::vector<const SequenceState*>& sequences,
                                   const std::vector<const float*>& queries_device,
                                   const std::vector<float*>& outputs_device,
                                   const std::vector<std::size_t>& query_tokens,
                                   std::size_t query_heads);

} // namespace kvflux::v2
