// Single-sequence PagedAttention dispatch (paged_attention's kernel side).
// One query token is a decode step and runs on the batch-decode kernel with
// a batch of one; several query tokens (a causal prefill or a multi-token
// suffix) run on the tcgen05 prefill kernel for 16-bit caches with
// head_size 128 and block 16, and on the generic kernel otherwise.
#include "common.cuh"
#include "launch.h"

namespace kvfx {

uint64_t attention_workspace_bytes(const CacheView& c, uint64_t query_tokens, uint64_t kv_tokens,
                                   uint32_t q_heads) {
    if (query_tokens == 1) return decode_workspace_bytes(c, 1, q_heads, kv_tokens, 0);
    return 0;
}

cudaError_t launch_attention(const CacheView& c, const AttentionArgs& a, unsigned* status,
                             cudaStream_t s) {
    if (a.query_tokens == 1 && decode_workspace_bytes(c, 1, a.q_heads, a.kv_tokens, 0) != 0) {
        DecodeArgs d{a.q, a.o, a.blocks, nullptr, 1, ceil_div(a.kv_tokens, c.bs), a.kv_tokens,
                     a.q_heads, 0, a.workspace, a.workspace_bytes};
        return launch_decode(c, d, status, s);
    }
    if (prefill_tc_supported(c, a)) return launch_prefill_tc(c, a, status, s);
    GenericAttnArgs g{a.q, a.o, a.blocks, 0, nullptr, a.query_tokens, a.kv_tokens, a.q_heads};
    return launch_attention_generic(c, g, status, s);
}

}  // namespace kvfx
