/*
 * kvoracle.h - CPU restatement of KVFlux's v2 paged-KV path.
 *
 * TEST INFRASTRUCTURE ONLY. The parity tests, the smoke check and the CPU
 * baseline of bench.py use this library as the checker; the product
 * (kvflux_b200) never links or calls it.
 *
 * Every function cites the reference code it restates (paths inside the
 * KVFlux repository). Element-type conversions are our own: bf16 -> f32 is a
 * 16-bit shift, f16 -> f32 decodes the IEEE half format exactly.
 */
#ifndef KVORACLE_H
#define KVORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KVO_OK 0
#define KVO_EINVAL 1
#define KVO_ERANGE 2
#define KVO_EOVERFLOW 3

/* dtype codes: 0 f16, 1 bf16, 2 f32 (same as kvflux::DType). */

/* Paged write of raw rows (src/v2/paged_kv_write.cu:72-81): for token i and
 * head h, row (slot_i / bs, h, slot_i % bs) of K/V <- row (i, h) of k_new/v_new.
 * Rows are row_bytes wide; slots are checked against num_blocks * bs. */
int kvo_write(uint8_t* k_cache, uint8_t* v_cache, uint64_t num_blocks, uint32_t heads, uint32_t bs,
              uint64_t row_bytes, const uint8_t* k_new, const uint8_t* v_new, const uint64_t* slots,
              uint64_t n);

/* Gather of one sequence (src/v2/paged_kv_read.cu:77-85). */
int kvo_gather(const uint8_t* k_cache, const uint8_t* v_cache, uint64_t num_blocks, uint32_t heads,
               uint32_t bs, uint64_t row_bytes, const uint64_t* blocks, uint64_t num_tokens,
               uint8_t* k_out, uint8_t* v_out);

/* Elementwise conversion of a cache-typed array to float. */
void kvo_to_f32(const void* src, int dtype, uint64_t count, float* dst);

/* reference_attention (src/v2/reference_attention.cpp:28-91): causal GQA
 * attention over contiguous FP32 Q/K/V with FP64 accumulation and the
 * three-pass softmax, same operation order. Q/O [Lq][Hq][hd], K/V [Lkv][Hkv][hd]. */
int kvo_reference_attention(const float* q, const float* k, const float* v, uint64_t q_tokens,
                            uint64_t kv_tokens, uint64_t q_heads, uint64_t kv_heads, uint64_t head_size,
                            float* out);

/* The reference's CPU path for batch decode: per request, gather its pages
 * (kvo_gather), convert to FP32, then kvo_reference_attention with one query
 * (the last position). Requests [first, first+count) are computed with
 * `threads` worker threads (requests are independent, so the result does not
 * depend on the thread count). table: [batch][max_blocks] page ids. */
int kvo_decode_batch(const uint8_t* k_cache, const uint8_t* v_cache, int dtype, uint64_t num_blocks,
                     uint32_t kv_heads, uint32_t bs, uint32_t head_size, const uint64_t* table,
                     uint64_t max_blocks, const uint64_t* lens, uint64_t first, uint64_t count,
                     uint32_t q_heads, const float* q, float* out, int threads);

/* One sequence, `q_tokens` queries aligned to the end of `kv_tokens`
 * (paged_attention's contract), computed for query rows [row_begin, row_end)
 * only (a row = one query token, all heads); rows outside are left untouched. */
int kvo_attention_rows(const uint8_t* k_cache, const uint8_t* v_cache, int dtype, uint64_t num_blocks,
                       uint32_t kv_heads, uint32_t bs, uint32_t head_size, const uint64_t* blocks,
                       uint64_t q_tokens, uint64_t kv_tokens, uint32_t q_heads, const float* q,
                       uint64_t row_begin, uint64_t row_end, float* out, int threads);

#ifdef __cplusplus
}
#endif

#endif /* KVORACLE_H */
