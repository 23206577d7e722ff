#pragma once
// CPU correctness oracle: softmax(Q K^T / sqrt(head_size) + causal mask) V
// over contiguous tensors, FP64 accumulation (reference:
// include/kvflux/v2/reference_attention.h:10-27). Q/O
// [query_tokens][query_heads][head_size], K/V [kv_tokens][kv_heads][head_size];
// Q is the suffix of the K/V sequence.
//
// A host function of libkvflux_b200 (as in KVFlux's library), for programs
// that check the GPU kernels against it; no GPU entry point calls it.
#include <cstddef>
#include <vector>

namespace kvflux::v2 {

struct AttentionShape {
    std::size_t query_tokens;
    std::size_t kv_tokens;
    std::size_t query_heads;
    std::size_t kv_heads;
    std::size_t head_size;
};

std::vector<float> reference_attention(const std::vector<float>& query,
                                       const std::vector<float>& key,
                                       const std::vector<float>& value,
                                       const AttentionShape& shape);

} // namespace kvflux::v2
