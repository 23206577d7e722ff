// Host-side declarations of the kernel launchers (internal to the library).
// Every launcher enqueues on `stream` and returns the launch's cudaError_t.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kvfx.h"

namespace kvfx {

__host__ __device__ constexpr uint64_t ceil_div(uint64_t a, uint64_t b) { return (a + b - 1) / b; }
__host__ __device__ constexpr uint64_t umin64(uint64_t a, uint64_t b) { return a < b ? a : b; }

// Validated, derived view of a kvfx_cache.
struct CacheView {
    char* k;
    char* v;
    uint64_t num_blocks;
    uint32_t heads, bs, hd, dtype, elem;
    uint64_t row_bytes;        // head_size * elem: one (token, head) row
    uint64_t chunk_bytes;      // block_size * row_bytes: one head of one page
    uint64_t page_bytes;       // heads * chunk_bytes
    uint64_t slot_count;       // num_blocks * block_size
    int device;
};

// Largest vector width in {16, 8, 4, 2, 1} bytes dividing `bytes` and every
// address in `ptrs` (n of them).
uint32_t vector_width(uint64_t bytes, const void* const* ptrs, int n);

cudaError_t launch_write(const CacheView& c, const void* k_new, const void* v_new,
                         const uint64_t* slots, uint64_t n, unsigned* status, cudaStream_t s);

cudaError_t launch_copy_page(const CacheView& c, uint64_t src, uint64_t dst, unsigned* status,
                             cudaStream_t s);

// Layer batches over caches of one shape (layers[0..num_layers), at most
// KVFX_MAX_LAYERS): layer l's new rows start at k_new + l * layer_stride bytes.
cudaError_t launch_write_layers(const CacheView* layers, uint32_t num_layers, const void* k_new,
                                const void* v_new, uint64_t layer_stride, const uint64_t* slots, uint64_t n,
                                unsigned* status, cudaStream_t s);

// Gather of `batch` sequences. If `per_seq_out` is false, k_out/v_out point to
// a single sequence's outputs (batch must be 1) and `single_blocks`/`single_len`
// describe it; otherwise k_out/v_out are device arrays of device pointers and
// the block table is row-major [batch][max_blocks].
struct GatherArgs {
    const uint64_t* blocks;    // [batch][max_blocks] (batch == 1: the one row)
    const uint64_t* lens;      // device lengths, or nullptr when batch == 1
    uint64_t single_len;       // length when lens == nullptr
    uint64_t batch, max_blocks;
    void* const* k_out_list;   // device array (batched) or nullptr
    void* const* v_out_list;
    void* k_out;               // single-sequence outputs
    void* v_out;
    uint64_t max_len;          // host bound of the lengths (grid sizing)
    uint64_t out_offset = 0;   // bytes added to every output pointer (SIMT kernel only)
    bool force_simt = false;   // take the element-wise kernel (needed for out_offset != 0)
};
cudaError_t launch_gather(const CacheView& c, const GatherArgs& a, unsigned* status, cudaStream_t s);
// Batched gather of every layer (a.k_out_list / a.v_out_list per sequence;
// layer l at + l * out_layer_stride bytes). Returns cudaErrorNotSupported for
// rows or alignments the 16-byte kernel cannot take (no launch).
cudaError_t launch_gather_layers(const CacheView* layers, uint32_t num_layers, const GatherArgs& a,
                                 uint64_t out_layer_stride, unsigned* status, cudaStream_t s);

struct DecodeArgs {
    const float* q;
    float* o;
    const uint64_t* table;
    const uint64_t* lens;
    uint64_t batch, max_blocks, max_len;
    uint32_t q_heads, pages_per_split;
    void* workspace;
    uint64_t workspace_bytes;
    // Append mode (kvfx_decode_append), all null for a plain decode: row b's
    // new token sits at position lens[b] - 1, its K/V rows are
    // k_new/v_new[b][h][:] (cache dtype) and its slot is new_slots[b]; the
    // launch writes them into the cache, stores the slot's page into
    // table_out[b][(lens[b] - 1) / bs] (table_out == table) and attends over
    // the updated rows.
    const void* k_new = nullptr;
    const void* v_new = nullptr;
    const uint64_t* new_slots = nullptr;
    uint64_t* table_out = nullptr;
};
// Decode workspace layout: the split counters first, then the split
// partials. The counters (16 bits each, one per (row, KV head) of the largest
// batch a launch takes) fill a region whose size depends only on the cache's
// KV heads, so a workspace zero-filled once stays usable for every batch and
// length: the launch that completes a counter's count resets it to zero.
constexpr uint64_t kDecodeCounterRows = 65536;
constexpr uint64_t decode_counter_bytes(uint32_t heads) {
    return (kDecodeCounterRows * heads * 2 + 255) & ~uint64_t(255);
}
uint64_t decode_workspace_bytes(const CacheView& c, uint64_t batch, uint32_t q_heads,
                                uint64_t max_len, uint32_t pages_per_split);
uint32_t decode_pages_per_split(const CacheView& c, uint64_t batch, uint32_t q_heads,
                                uint64_t max_len, uint64_t total_tokens);
cudaError_t launch_decode(const CacheView& c, const DecodeArgs& a, unsigned* status, cudaStream_t s);

struct AttentionArgs {
    const float* q;
    float* o;
    const uint64_t* blocks;
    uint64_t query_tokens, kv_tokens;
    uint32_t q_heads;
    void* workspace;
    uint64_t workspace_bytes;
};
uint64_t attention_workspace_bytes(const CacheView& c, uint64_t query_tokens, uint64_t kv_tokens,
                                   uint32_t q_heads);
cudaError_t launch_attention(const CacheView& c, const AttentionArgs& a, unsigned* status,
                             cudaStream_t s);
// Causal prefill on tcgen05 (prefill.cu): shapes it covers, and the launch.
bool prefill_tc_supported(const CacheView& c, const AttentionArgs& a);
cudaError_t launch_prefill_tc(const CacheView& c, const AttentionArgs& a, unsigned* status, cudaStream_t s);
// Several sequences (each prefill_tc_supported, one q_heads) in one
// persistent launch; at most KVFX_MAX_PREFILL_SEQS.
cudaError_t launch_prefill_tc_batch(const CacheView& c, const AttentionArgs* seqs, uint32_t n, unsigned* status,
                                    cudaStream_t s);

// Generic SIMT attention over "query rows" (used by both entry points for the
// shapes the specialised kernels do not cover).
struct GenericAttnArgs {
    const float* q;
    float* o;
    const uint64_t* blocks;     // row-major table, row stride `row_stride`
    uint64_t row_stride;        // 0: every query row uses row 0 (single sequence)
    const uint64_t* lens;       // batch mode: device lengths, one query per sequence
    uint64_t units;             // batch size, or query_tokens for a single sequence
    uint64_t kv_tokens;         // single-sequence mode: sequence length
    uint32_t q_heads;
};
cudaError_t launch_attention_generic(const CacheView& c, const GenericAttnArgs& a,
                                     unsigned* status, cudaStream_t s);

// Tensor maps over the K and V caches for the TMA-fed kernels (cached per cache).
struct CacheMaps {
    CUtensorMap k;
    CUtensorMap v;
    bool valid;
};
const CacheMaps* cache_maps(const CacheView& c, cudaError_t* err);
// Unswizzled maps over the K and V caches, one box = one (page, head) tile of
// block_size rows (the TMA gather's loads; cached per cache).
const CacheMaps* gather_maps(const CacheView& c, cudaError_t* err);
// Encodes a tiled, unswizzled tensor map (dims and box innermost first,
// strides in bytes for dims 1..rank-1).
bool encode_tiled(CUtensorMap* map, CUtensorMapDataType type, uint32_t rank, void* base, const uint64_t* dims,
                  const uint64_t* strides, const uint32_t* box, cudaError_t* err);

// The batch-decode fast path with caller-provided tensor maps (16-bit caches,
// head_size 64/128, block 16, group <= 8 only).
cudaError_t launch_decode_with_maps(const CacheView& c, const DecodeArgs& a, const CacheMaps& maps,
                                    unsigned* status, cudaStream_t s);
// Runs the bounded-wait self-test kernel and waits for it; completed[w] = 1 if
// warp w's wait completed, 0 if it gave up (the expected outcome).
cudaError_t launch_wait_selftest(unsigned* status, cudaStream_t s, int* completed);

// Flags raised by kvfx_decode_noalloc's launches on `device` (its own status
// word, a device variable); cleared when `clear`. False on a CUDA error.
bool noalloc_status(int device, unsigned* flags, bool clear);

// Records the calling thread's message for kvfx_last_error().
void set_last_error(const char* msg);

int device_sm_count(int device);

}  // namespace kvfx
