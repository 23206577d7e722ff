// ref_gpu_shim.cpp - one C entry point over the reference's own GPU path.
//
// TEST INFRASTRUCTURE ONLY. oracle/build.py compiles this file with nvcc
// (sm_100a) together with KVFlux's own sources where they lie - its CPU
// control plane, the v1 GpuMemoryPool, the v2 PagedKVStorage and its CUDA
// write, read and attention files (src/v2/paged_kv_write.cu,
// src/v2/paged_kv_read.cu, src/v2/paged_attention.cu) - into
// oracle/_ref/libkvflux_ref_gpu.so. Only the function below is exported
// (-fvisibility=hidden), so the reference's kvflux:: symbols never clash with
// the product library's.
//
// Use: the reference's unmodified GPU kernels, driven through its public API
// on the same B200 and the same inputs, as a GPU-side baseline (bench.py) and
// as an independent parity check of this build's batch decode (tests).
#include <cuda_runtime_api.h>

#include <algorithm>
#include <chrono>
#include <cstdint>
#include <memory>
#include <stdexcept>
#include <vector>

#include "kvflux/physical_block_pool.h"
#include "kvflux/v2/paged_attention.h"
#include "kvflux/v2/paged_kv_storage.h"
#include "kvflux/v2/paged_kv_write.h"
#include "kvflux/v2/sequence_state.h"
#include "kvflux/v2/slot_mapping.h"

#define REF_API extern "C" __attribute__((visibility("default")))

namespace {

struct DeviceBuffer {
    void* p = nullptr;
    explicit DeviceBuffer(std::size_t bytes) {
        if (cudaMalloc(&p, bytes) != cudaSuccess) throw std::runtime_error("cudaMalloc");
    }
    ~DeviceBuffer() {
        if (p) (void)cudaFree(p);
    }
};

double median(std::vector<double> v) {
    std::sort(v.begin(), v.end());
    return v[v.size() / 2];
}

}  // namespace

// Batch decode through the reference's public API on `device`:
//  - a PhysicalBlockPool of num_blocks pages of block_size tokens whose free
//    list hands out page ids in `page_order` (every page allocated, then freed
//    in reverse order of page_order);
//  - a PagedKVStorage (kv_heads x head_size, dtype 0 f16 / 1 bf16 / 2 f32);
//  - `batch` sequences of lens[b] tokens, appended in order;
//  - every token's K/V rows (host, [sum(lens)][kv_heads][head_size], in
//    sequence order) written with write_paged_kv in one call, timed, then
//    the same call `reps` more times (same slots and rows), timed each;
//  - paged_attention_batch with Q (host [batch][q_heads][head_size]) run
//    `reps` times (each call synchronous, as the reference's API is; timed
//    with a host steady clock around each call).
// Writes O (host) and the times in milliseconds: write_ms[0] the first
// write, write_ms[1] the median of the repeats, decode_ms the median decode.
// Returns 0, or 1 on any exception (message not kept).
REF_API int kvref_gpu_decode(int device, uint64_t num_blocks, uint32_t block_size, const uint64_t* page_order,
                             uint32_t kv_heads, uint32_t q_heads, uint32_t head_size, uint32_t dtype,
                             const uint64_t* lens, uint64_t batch, const void* k_rows, const void* v_rows,
                             const float* q, float* o, int reps, double* write_ms, double* decode_ms) {
    try {
        if (cudaSetDevice(device) != cudaSuccess) return 1;
        kvflux::PhysicalBlockPool pool(num_blocks, block_size);
        std::vector<kvflux::PhysicalBlockHandle> held;
        held.reserve(num_blocks);
        for (uint64_t i = 0; i < num_blocks; ++i) held.push_back(pool.allocate());
        for (uint64_t i = num_blocks; i-- > 0;) pool.free(held[page_order[i]]);
        const auto dt = dtype == 0 ? kvflux::DType::Float16 : dtype == 1 ? kvflux::DType::BFloat16
                                                                         : kvflux::DType::Float32;
        kvflux::v2::PagedKVStorage storage(pool, kv_heads, head_size, dt, device);
        std::vector<std::unique_ptr<kvflux::v2::SequenceState>> seqs;
        std::vector<kvflux::v2::TokenWrite> writes;
        uint64_t total = 0;
        for (uint64_t b = 0; b < batch; ++b) {
            seqs.push_back(std::make_unique<kvflux::v2::SequenceState>(b + 1, pool));
            seqs.back()->append_tokens(lens[b]);
            for (uint64_t t = 0; t < lens[b]; ++t) writes.push_back({seqs.back().get(), t});
            total += lens[b];
        }
        const kvflux::v2::SlotMapping slots = kvflux::v2::build_slot_mapping(writes);
        const std::size_t elem = dtype == 2 ? 4 : 2;
        const std::size_t kv_bytes = total * kv_heads * head_size * elem;
        DeviceBuffer dk(kv_bytes), dv(kv_bytes);
        if (cudaMemcpy(dk.p, k_rows, kv_bytes, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(dv.p, v_rows, kv_bytes, cudaMemcpyHostToDevice) != cudaSuccess)
            return 1;
        std::vector<double> wtimes;
        for (int i = 0; i <= std::max(reps, 1); ++i) {
            const auto t0 = std::chrono::steady_clock::now();
            kvflux::v2::write_paged_kv(storage, dk.p, dv.p, slots);
            wtimes.push_back(
                std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count());
        }
        write_ms[0] = wtimes[0];
        write_ms[1] = median(std::vector<double>(wtimes.begin() + 1, wtimes.end()));
        auto t0 = std::chrono::steady_clock::now();

        const std::size_t q_bytes = batch * q_heads * head_size * sizeof(float);
        DeviceBuffer dq(q_bytes), dout(q_bytes);
        if (cudaMemcpy(dq.p, q, q_bytes, cudaMemcpyHostToDevice) != cudaSuccess) return 1;
        std::vector<const kvflux::v2::SequenceState*> view;
        for (auto& s : seqs) view.push_back(s.get());
        std::vector<double> times;
        for (int i = 0; i < std::max(reps, 1); ++i) {
            t0 = std::chrono::steady_clock::now();
            kvflux::v2::paged_attention_batch(storage, view, static_cast<const float*>(dq.p),
                                              static_cast<float*>(dout.p), q_heads);
            times.push_back(
                std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count());
        }
        *decode_ms = median(times);
        if (cudaMemcpy(o, dout.p, q_bytes, cudaMemcpyDeviceToHost) != cudaSuccess) return 1;
        seqs.clear();
        return 0;
    } catch (...) {
        return 1;
    }
}
