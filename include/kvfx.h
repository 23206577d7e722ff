/*
 * kvfx.h - C ABI of the B200 (sm_100a) paged-KV data path.
 *
 * Plain pointers and sizes only: no C++ or torch types cross this boundary, so
 * any FFI (ctypes, cgo, JNI, N-API) can bind it. Every entry point is
 * stream-ordered: it enqueues work on `stream` (a cudaStream_t; NULL is the
 * legacy default stream) and returns without synchronising. Device arrays
 * must be resident on `cache->device`. Return value: KVFX_OK or an error code;
 * kvfx_last_error() gives a message for the calling thread's last failure.
 *
 * The cache layout is the reference's single-layer paged layout
 * (src/v2/paged_kv_layout.cpp:27-68 in KVFlux):
 *     K[num_blocks][num_kv_heads][block_size][head_size], then V alike,
 * and a slot id is physical_block * block_size + offset_in_block
 * (src/v2/slot_mapping.cpp:29).
 *
 * These entry points trust the tables they are given only as far as memory
 * safety: a slot or block id at or beyond the cache is skipped (writes) or
 * read as nothing, and sets KVFX_FLAG_BAD_INDEX in the device status word
 * (kvfx_device_status). The C++ API in include/kvflux/v2 validates everything
 * on the host first and raises the reference's exception types.
 */
#ifndef KVFX_H
#define KVFX_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes. */
#define KVFX_OK 0
#define KVFX_EINVAL 1       /* bad argument: null pointer, bad shape or dtype   */
#define KVFX_ERANGE 2       /* index outside the cache                           */
#define KVFX_EOVERFLOW 3    /* size arithmetic overflow                          */
#define KVFX_ECUDA 4        /* CUDA runtime error (message in kvfx_last_error)   */
#define KVFX_ETIMEOUT 5     /* a bounded device-side wait gave up                */
#define KVFX_ENOSPACE 6     /* workspace smaller than the *_workspace_bytes size */

/* Cache element types (same order as kvflux::DType). */
#define KVFX_F16 0
#define KVFX_BF16 1
#define KVFX_F32 2

/* Most layers one kvfx_write_layers / kvfx_gather_layers call takes. */
#define KVFX_MAX_LAYERS 128u

/* Most sequences one kvfx_attention_batch call takes. */
#define KVFX_MAX_PREFILL_SEQS 32u

/* Bits of the per-device status word. */
#define KVFX_FLAG_BAD_INDEX 1u  /* a slot/block id beyond the cache was skipped */
#define KVFX_FLAG_TIMEOUT 2u    /* a bounded wait inside a kernel expired        */

typedef struct kvfx_cache {
    void* k_base;            /* device address of K[0][0][0][0]                  */
    void* v_base;            /* device address of V[0][0][0][0]                  */
    uint64_t num_blocks;     /* physical pages                                   */
    uint32_t num_kv_heads;
    uint32_t block_size;     /* tokens per page                                  */
    uint32_t head_size;
    uint32_t dtype;          /* KVFX_F16 / KVFX_BF16 / KVFX_F32                  */
    int32_t device;          /* CUDA ordinal holding the cache                   */
    uint32_t reserved;       /* must be 0                                        */
} kvfx_cache;

/*
 * Paged KV write: for token i, K[slot_i / bs][h][slot_i % bs][:] = k_new[i][h][:]
 * and the same for V, for all h. k_new/v_new: [num_tokens][num_kv_heads][head_size]
 * in the cache dtype; slots: device uint64[num_tokens], pairwise distinct.
 * Replaces the kernel launch of write_paged_kv (KVFlux src/v2/paged_kv_write.cu:86-97).
 */
int kvfx_write(const kvfx_cache* cache, const void* k_new, const void* v_new,
               const uint64_t* slots, uint64_t num_tokens, void* stream);

/*
 * Gather of one sequence: k_out[t][h][:] = K[blocks[t / bs]][h][t % bs][:] for
 * t < num_tokens (V alike). blocks: device uint64[ceil(num_tokens / bs)].
 * Outputs must not overlap each other or the cache. Rows that are 16-byte
 * multiples of at most 256 elements, with 16-byte aligned bases, move by TMA
 * tensor copies (one load and one store per page and KV head); other shapes
 * by vector loads and stores.
 * Replaces the kernel launch of read_paged_kv (KVFlux src/v2/paged_kv_read.cu:90-102).
 */
int kvfx_gather(const kvfx_cache* cache, const uint64_t* blocks, uint64_t num_tokens,
                void* k_out, void* v_out, void* stream);

/*
 * Batched gather: sequence b has seq_lens[b] tokens, pages in row b of the
 * row-major table blocks[batch][max_blocks_per_seq], and outputs k_out[b] /
 * v_out[b] (device arrays of device pointers). One launch for the whole batch.
 * No counterpart in the reference, which gathers one sequence per call.
 */
int kvfx_gather_batch(const kvfx_cache* cache, const uint64_t* blocks,
                      const uint64_t* seq_lens, uint64_t batch, uint64_t max_blocks_per_seq,
                      void* const* k_out, void* const* v_out, void* stream);

/*
 * Layer batches. A model keeps one cache per layer, all with one shape and
 * one page pool (the reference's multi-layer plan: one PagedKVStorage per
 * layer over one PhysicalBlockPool, docs/v2_paged_kv_storage.md:19), so a
 * slot or a page id means the same place in every layer. These two calls
 * move one step's rows (or a batch of sequences) for every layer in one
 * launch, e.g. the whole KV of a request arriving from a prefill instance or
 * leaving for host memory. caches: host array of num_layers (<=
 * KVFX_MAX_LAYERS) descriptors equal in all fields but k_base and v_base.
 * No counterpart in the reference, which writes and reads one layer per call.
 */

/* kvfx_write on every layer: layer l's rows are k_new/v_new + l * layer_stride_bytes
 * ([num_tokens][num_kv_heads][head_size] each; layer_stride_bytes >= that size). */
int kvfx_write_layers(const kvfx_cache* caches, uint32_t num_layers, const void* k_new,
                      const void* v_new, uint64_t layer_stride_bytes, const uint64_t* slots,
                      uint64_t num_tokens, void* stream);

/* kvfx_gather_batch on every layer: sequence b's layer l goes to
 * k_out[b] + l * out_layer_stride_bytes (and v_out alike). */
int kvfx_gather_layers(const kvfx_cache* caches, uint32_t num_layers, const uint64_t* blocks,
                       const uint64_t* seq_lens, uint64_t batch, uint64_t max_blocks_per_seq,
                       void* const* k_out, void* const* v_out, uint64_t out_layer_stride_bytes,
                       void* stream);

/*
 * Whole-page copy of K and V from src_block to dst_block (byte-exact).
 * Replaces the two cudaMemcpyAsync of PagedKVStorage::copy_block
 * (KVFlux src/v2/paged_kv_storage.cpp:70-93).
 */
int kvfx_copy_page(const kvfx_cache* cache, uint64_t src_block, uint64_t dst_block,
                   void* stream);

/*
 * Batch decode PagedAttention: one last-position query per sequence.
 *   q, o         : device float[batch][q_heads][head_size]
 *   block_table  : device uint64[batch][max_blocks_per_seq], row b holds the
 *                  pages of sequence b (entries past its length are not read)
 *   seq_lens     : device uint64[batch], each in [1, max_seq_len]
 *   max_seq_len  : host-side upper bound of seq_lens (sizes the grid)
 *   pages_per_split: split-K chunk in pages; 0 chooses one from the shape
 *   workspace    : device scratch of kvfx_decode_workspace_bytes(...) bytes,
 *                  zero-filled (cudaMemset) before its first use. Its start
 *                  holds the split counters, which every launch leaves at
 *                  zero again, so it stays ready for the next launch of any
 *                  batch, lengths or split size on caches with the same
 *                  num_kv_heads (zero it again before using it with a cache
 *                  of another head count). Launches that share a workspace
 *                  must not overlap on the GPU.
 * q_heads must be a multiple of num_kv_heads; Q head j uses KV head
 * j / (q_heads / num_kv_heads). Scale 1/sqrt(head_size).
 * Replaces paged_attention_batch's launch (KVFlux src/v2/paged_attention.cu:248-313).
 */
uint64_t kvfx_decode_workspace_bytes(const kvfx_cache* cache, uint64_t batch,
                                     uint32_t q_heads, uint64_t max_seq_len,
                                     uint32_t pages_per_split);
uint32_t kvfx_decode_pages_per_split(const kvfx_cache* cache, uint64_t batch,
                                     uint32_t q_heads, uint64_t max_seq_len,
                                     uint64_t total_tokens);
int kvfx_decode(const kvfx_cache* cache, const float* q, float* o,
                const uint64_t* block_table, const uint64_t* seq_lens, uint64_t batch,
                uint64_t max_blocks_per_seq, uint32_t q_heads, uint64_t max_seq_len,
                uint32_t pages_per_split, void* workspace, uint64_t workspace_bytes,
                void* stream);

/*
 * One batch decode step fused with its paged KV write. Row b's new token is
 * position seq_lens[b] - 1 (seq_lens already count it); its K/V rows are
 * k_new/v_new[b][num_kv_heads][head_size] in the cache dtype and its slot is
 * new_slots[b] (device uint64[batch]), whose offset in its page must equal
 * (seq_lens[b] - 1) % block_size. The launch writes those rows into the cache,
 * stores the slot's page into block_table[b][(seq_lens[b] - 1) / block_size]
 * (block_table is device memory that stays resident between steps; entries
 * before that column are read as they are), and computes the same attention
 * as kvfx_decode over the updated rows; q, o, workspace and the other
 * arguments as for kvfx_decode. A slot outside the cache or at the wrong
 * offset is not written and sets KVFX_FLAG_BAD_INDEX. Each new slot must lie
 * in a page that no other row of the launch reads (copy a shared last page on
 * write first, as append_token_cow does); rows' slots must be distinct.
 * Replaces, for a batch, the write_paged_kv + paged_attention pair of the
 * reference's decode step (KVFlux src/v2/sequence_lifecycle.cpp:53-73), with
 * the block table kept on the device instead of uploaded per call
 * (src/v2/paged_attention.cu:287-292).
 */
int kvfx_decode_append(const kvfx_cache* cache, const void* k_new, const void* v_new,
                       const uint64_t* new_slots, const float* q, float* o, uint64_t* block_table,
                       const uint64_t* seq_lens, uint64_t batch, uint64_t max_blocks_per_seq,
                       uint32_t q_heads, uint64_t max_seq_len, uint32_t pages_per_split,
                       void* workspace, uint64_t workspace_bytes, void* stream);

/*
 * Batch decode that allocates nothing: the same computation and arguments as
 * kvfx_decode without pages_per_split and the workspace. No counterpart in
 * the reference. For callers that cannot call cudaMalloc: engines that hand
 * all device memory to their KV pool at start-up, loops that cannot take
 * cudaMalloc/cudaFree's implicit synchronisation, and embedders whose
 * allocator policy forbids device allocations outside their own allocator.
 * Its scratch (split-K partials + counters) is a static 16 MiB device array
 * held by every GPU that loads this code until the process exits; the split
 * size is chosen so the scratch fits, and a batch whose batch x num_kv_heads
 * cannot fit even with one split per sequence is rejected with KVFX_ENOSPACE.
 * The first call on a device looks up the array's address (make it before
 * any stream capture; a device reset invalidates it, so do not call this on
 * a device after resetting it). All calls share the array: calls that
 * overlap on the GPU race. The split counters return to zero at the end of
 * every launch; the first call on a device, and a call whose cache has
 * another num_kv_heads than the previous call's, clears them on `stream`
 * first. Device-side flags (an out-of-range page id, a bounded wait that
 * gave up) are kept in a device variable that kvfx_device_status reads
 * together with the other kernels' flags.
 */
int kvfx_decode_noalloc(const kvfx_cache* cache, const float* q, float* o,
                        const uint64_t* block_table, const uint64_t* seq_lens, uint64_t batch,
                        uint64_t max_blocks_per_seq, uint32_t q_heads, uint64_t max_seq_len,
                        void* stream);

/*
 * Single-sequence causal PagedAttention with query_tokens queries aligned to
 * the end of the kv_tokens-long sequence (query i sees positions
 * <= kv_tokens - query_tokens + i). q, o: device float[query_tokens][q_heads][head_size];
 * blocks: device uint64[ceil(kv_tokens / bs)]. workspace: as for kvfx_decode
 * (zero-filled before its first use; query_tokens == 1 runs the decode
 * kernel, the only case that needs one).
 * Replaces paged_attention's launch (KVFlux src/v2/paged_attention.cu:193-246).
 */
uint64_t kvfx_attention_workspace_bytes(const kvfx_cache* cache, uint64_t query_tokens,
                                        uint64_t kv_tokens, uint32_t q_heads);
int kvfx_attention(const kvfx_cache* cache, const float* q, float* o, const uint64_t* blocks,
                   uint64_t query_tokens, uint64_t kv_tokens, uint32_t q_heads,
                   void* workspace, uint64_t workspace_bytes, void* stream);

/*
 * kvfx_attention over num_seqs (<= KVFX_MAX_PREFILL_SEQS) sequences of one
 * cache in one call: sequence i has query_tokens[i] queries aligned to the
 * end of its kv_tokens[i] tokens, Q and O at the device addresses q[i] and
 * o[i] (float[query_tokens[i]][q_heads][head_size]) and its pages in row i of
 * the device table block_table[num_seqs][max_blocks_per_seq]. q, o,
 * query_tokens and kv_tokens are host arrays of num_seqs entries. Each
 * output equals what kvfx_attention gives for that sequence alone (bit for
 * bit); the sequences of tensor-core prefill shapes run as one persistent
 * launch that deals the query tiles of all of them, heaviest first, over the
 * SMs, the others as one kvfx_attention each after it. The workspace is the largest
 * kvfx_attention_workspace_bytes of the sequences. Sequences with no queries
 * are skipped. Replaces the per-sequence loop over paged_attention's launch
 * (KVFlux src/v2/paged_attention.cu:193-246) that a batched prefill makes.
 */
int kvfx_attention_batch(const kvfx_cache* cache, uint32_t num_seqs, const float* const* q, float* const* o,
                         const uint64_t* block_table, uint64_t max_blocks_per_seq,
                         const uint64_t* query_tokens, const uint64_t* kv_tokens, uint32_t q_heads,
                         void* workspace, uint64_t workspace_bytes, void* stream);

/* Message of the calling thread's last failed call ("" if none). */
const char* kvfx_last_error(void);

/*
 * Reads the status word of `device` (KVFX_FLAG_* bits set by kernels since
 * the last clear, kvfx_decode_noalloc's included) after the caller has
 * synchronised the work in question; clears it when `clear` is non-zero.
 */
int kvfx_device_status(int device, uint32_t* flags, int clear);

/*
 * Self-test of device-side failure detection. Every kernel here that waits on
 * a shared-memory barrier (TMA arrivals, tensor-core commits) bounds the wait
 * (2 s): a wait that runs out raises KVFX_FLAG_TIMEOUT in the status word and
 * the kernel returns instead of hanging; the C++ API then throws
 * std::runtime_error. This call runs those waits (inline and out-of-line
 * forms) on `device` on a barrier that nothing completes and nothing is in
 * flight on, synchronously (~2 s). Returns KVFX_ETIMEOUT when both waits gave
 * up and reported it (the expected outcome; the context stays usable),
 * KVFX_EINVAL if a wait did not report it, KVFX_ECUDA on a CUDA error. The
 * status word is left as it was (run no other work on the device meanwhile,
 * or its timeout flag may be folded into the test's). No counterpart in the reference, whose
 * kernels do not wait on barriers.
 */
int kvfx_selftest_wait_timeout(int device);

/* Library version, e.g. "kvflux-b200 0.1.0 sm_100a". */
const char* kvfx_version(void);

#ifdef __cplusplus
}
#endif

#endif /* KVFX_H */
