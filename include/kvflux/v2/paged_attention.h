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

} // namespace kvflux::v2
