// ref_shim.cpp - C entry points over the reference's own CPU sources.
//
// TEST INFRASTRUCTURE ONLY. oracle/build.py compiles this file together with
// KVFlux's CPU sources where they lie (src/block_manager.cpp,
// src/physical_block_pool.cpp, src/v2/{block_table,sequence_state,
// batch_block_table,slot_mapping,paged_kv_layout,reference_attention,
// prefix_cache,paged_kv_read_table}.cpp) into oracle/_ref/libkvflux_ref.so.
// Only the functions below are exported (-fvisibility=hidden), so the
// reference's kvflux:: symbols never clash with the product library's.
//
// Uses: A/B checks of the re-implemented control plane (same op script, same
// page ids), bit-exact checks of oracle/kvoracle.c's reference_attention, and
// bench.py's reference arm (the reference's own reference_attention on the
// host cores, one std::thread per request slice).
#include <cmath>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <thread>
#include <vector>

#include "kvflux/physical_block_pool.h"
#include "kvflux/v2/batch_block_table.h"
#include "kvflux/v2/reference_attention.h"
#include "kvflux/v2/sequence_state.h"
#include "kvflux/v2/slot_mapping.h"

#define REF_API extern "C" __attribute__((visibility("default")))

namespace {

int code_of(const std::exception& e) {
    if (dynamic_cast<const kvflux::CapacityError*>(&e)) return 5;
    if (dynamic_cast<const std::invalid_argument*>(&e)) return 1;
    if (dynamic_cast<const std::out_of_range*>(&e)) return 2;
    if (dynamic_cast<const std::overflow_error*>(&e)) return 3;
    if (dynamic_cast<const std::logic_error*>(&e)) return 4;
    return 6;
}

template <typename F>
int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        return code_of(e);
    }
}

float bf16_to_f32(uint16_t h) {
    uint32_t bits = static_cast<uint32_t>(h) << 16;
    float f;
    std::memcpy(&f, &bits, sizeof f);
    return f;
}

}  // namespace

// ------------------------------------------------------------ control plane

REF_API void* ref_pool_new(uint64_t capacity, uint64_t block_size) {
    try {
        return new kvflux::PhysicalBlockPool(capacity, block_size);
    } catch (...) {
        return nullptr;
    }
}
REF_API void ref_pool_delete(void* p) { delete static_cast<kvflux::PhysicalBlockPool*>(p); }
REF_API int ref_pool_allocate(void* p, uint64_t* id, uint64_t* gen) {
    return guarded([&] {
        const auto h = static_cast<kvflux::PhysicalBlockPool*>(p)->allocate();
        *id = h.id;
        *gen = h.generation;
    });
}
REF_API int ref_pool_free(void* p, uint64_t id, uint64_t gen) {
    return guarded([&] { static_cast<kvflux::PhysicalBlockPool*>(p)->free({id, gen}); });
}
REF_API int ref_pool_retain(void* p, uint64_t id, uint64_t gen) {
    return guarded([&] { static_cast<kvflux::PhysicalBlockPool*>(p)->retain({id, gen}); });
}
REF_API uint64_t ref_pool_available(void* p) { return static_cast<kvflux::PhysicalBlockPool*>(p)->available(); }
REF_API int ref_pool_ref_count(void* p, uint64_t id, uint64_t gen, uint64_t* out) {
    return guarded([&] { *out = static_cast<kvflux::PhysicalBlockPool*>(p)->ref_count({id, gen}); });
}

REF_API void* ref_seq_new(void* pool, uint64_t request_id) {
    return new kvflux::v2::SequenceState(request_id, *static_cast<kvflux::PhysicalBlockPool*>(pool));
}
REF_API void ref_seq_delete(void* s) { delete static_cast<kvflux::v2::SequenceState*>(s); }
REF_API int ref_seq_append_tokens(void* s, uint64_t n) {
    return guarded([&] { static_cast<kvflux::v2::SequenceState*>(s)->append_tokens(n); });
}
REF_API int ref_seq_append_token(void* s, uint64_t* block, uint64_t* offset) {
    return guarded([&] {
        const auto loc = static_cast<kvflux::v2::SequenceState*>(s)->append_token();
        *block = loc.physical_block;
        *offset = loc.offset_in_block;
    });
}
REF_API void* ref_seq_fork(void* s, uint64_t request_id) {
    try {
        return new kvflux::v2::SequenceState(static_cast<kvflux::v2::SequenceState*>(s)->fork_shared(request_id));
    } catch (...) {
        return nullptr;
    }
}
// Copy-on-write append with a recording copier (no data moves on the CPU).
REF_API int ref_seq_append_token_with_copy(void* s, uint64_t* block, uint64_t* offset, uint64_t* copied_from,
                                           uint64_t* copied_to) {
    *copied_from = *copied_to = UINT64_MAX;
    return guarded([&] {
        const auto loc = static_cast<kvflux::v2::SequenceState*>(s)->append_token_with_copy(
            [&](kvflux::PhysicalBlockHandle a, kvflux::PhysicalBlockHandle b) {
                *copied_from = a.id;
                *copied_to = b.id;
            });
        *block = loc.physical_block;
        *offset = loc.offset_in_block;
    });
}
REF_API uint64_t ref_seq_num_tokens(void* s) { return static_cast<kvflux::v2::SequenceState*>(s)->num_tokens(); }
REF_API uint64_t ref_seq_num_blocks(void* s) {
    return static_cast<kvflux::v2::SequenceState*>(s)->num_allocated_blocks();
}
REF_API int ref_seq_block_ids(void* s, uint64_t* out) {
    return guarded([&] {
        auto* seq = static_cast<kvflux::v2::SequenceState*>(s);
        for (std::size_t i = 0; i < seq->num_allocated_blocks(); ++i) out[i] = seq->physical_block_id(i);
    });
}
REF_API int ref_slot_mapping(void* const* seqs, const uint64_t* positions, uint64_t n, uint64_t* out) {
    return guarded([&] {
        std::vector<kvflux::v2::TokenWrite> batch;
        for (uint64_t i = 0; i < n; ++i) {
            batch.push_back({static_cast<const kvflux::v2::SequenceState*>(seqs[i]), positions[i]});
        }
        const auto slots = kvflux::v2::build_slot_mapping(batch);
        std::memcpy(out, slots.data(), slots.size() * sizeof(uint64_t));
    });
}
// Writes max_blocks first; table_out must hold n * max_blocks entries (call
// once with table_out == nullptr to learn max_blocks).
REF_API int ref_batch_table(void* const* seqs, uint64_t n, uint64_t* max_blocks, uint64_t* table_out,
                            uint64_t* lens_out) {
    return guarded([&] {
        std::vector<const kvflux::v2::SequenceState*> v;
        for (uint64_t i = 0; i < n; ++i) v.push_back(static_cast<const kvflux::v2::SequenceState*>(seqs[i]));
        const auto t = kvflux::v2::build_batch_block_table(v);
        *max_blocks = t.max_blocks_per_sequence();
        if (table_out != nullptr) {
            std::memcpy(table_out, t.block_table().data(), t.block_table().size() * sizeof(uint64_t));
            std::memcpy(lens_out, t.sequence_lengths().data(), t.sequence_lengths().size() * sizeof(uint64_t));
        }
    });
}

// ---------------------------------------------------------------- attention

REF_API int ref_reference_attention(const float* q, const float* k, const float* v, uint64_t q_tokens,
                                    uint64_t kv_tokens, uint64_t q_heads, uint64_t kv_heads, uint64_t head_size,
                                    float* out) {
    return guarded([&] {
        const std::size_t qn = q_tokens * q_heads * head_size, kn = kv_tokens * kv_heads * head_size;
        std::vector<float> qv(q, q + qn), kv(k, k + kn), vv(v, v + kn);
        const auto o = kvflux::v2::reference_attention(qv, kv, vv, {q_tokens, kv_tokens, q_heads, kv_heads, head_size});
        std::memcpy(out, o.data(), o.size() * sizeof(float));
    });
}

// The reference's CPU path for batch decode on bf16/f16/f32 caches: per
// request, gather its pages (the reference has no CPU gather; this restates
// src/v2/paged_kv_read.cu:77-85), widen to FP32 and call the reference's own
// reference_attention with one query. Requests [first, first+count) are split
// over `threads` std::threads.
REF_API int ref_decode_batch(const void* k_cache, const void* v_cache, int dtype, uint64_t num_kv_heads,
                             uint64_t block_size, uint64_t head_size, const uint64_t* table, uint64_t max_blocks,
                             const uint64_t* lens, uint64_t first, uint64_t count, uint64_t q_heads, const float* q,
                             float* out, int threads) {
    if (threads < 1) threads = 1;
    const uint64_t elem = dtype == 2 ? 4 : 2;
    auto widen = [&](const void* base, uint64_t index) -> float {
        if (dtype == 2) return static_cast<const float*>(base)[index];
        const uint16_t h = static_cast<const uint16_t*>(base)[index];
        if (dtype == 1) return bf16_to_f32(h);
        // f16: exact widening via the compiler's _Float16
        _Float16 x;
        std::memcpy(&x, &h, sizeof h);
        return static_cast<float>(x);
    };
    (void)elem;
    std::vector<int> status(threads, 0);
    auto work = [&](int t) {
        status[t] = guarded([&] {
            for (uint64_t r = first + t; r < first + count; r += threads) {
                const uint64_t len = lens[r];
                std::vector<float> kk(len * num_kv_heads * head_size), vv(kk.size());
                for (uint64_t tok = 0; tok < len; ++tok) {
                    const uint64_t page = table[r * max_blocks + tok / block_size];
                    for (uint64_t h = 0; h < num_kv_heads; ++h) {
                        const uint64_t src = ((page * num_kv_heads + h) * block_size + tok % block_size) * head_size;
                        const uint64_t dst = (tok * num_kv_heads + h) * head_size;
                        for (uint64_t d = 0; d < head_size; ++d) {
                            kk[dst + d] = widen(k_cache, src + d);
                            vv[dst + d] = widen(v_cache, src + d);
                        }
                    }
                }
                std::vector<float> qq(q + r * q_heads * head_size, q + (r + 1) * q_heads * head_size);
                const auto o = kvflux::v2::reference_attention(qq, kk, vv, {1, len, q_heads, num_kv_heads, head_size});
                std::memcpy(out + r * q_heads * head_size, o.data(), o.size() * sizeof(float));
            }
        });
    };
    std::vector<std::thread> pool;
    for (int t = 1; t < threads; ++t) pool.emplace_back(work, t);
    work(0);
    for (auto& th : pool) th.join();
    for (int s : status) {
        if (s != 0) return s;
    }
    return 0;
}
