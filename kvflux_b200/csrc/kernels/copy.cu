// Byte-moving kernels of the paged-KV data path: the slot-mapped write
// (kernel 1), the block-table gather (kernel 2) and the whole-page copy used
// by copy-on-write. All three are HBM-bound bit copies, so they move 16-byte
// vectors (or TMA bulk copies) and never interpret the element type.
//
// Index math follows the reference kernels:
//   write  K[(slot / bs * H + h) * bs + slot % bs][d] = K_new[i][h][d]
//          (KVFlux src/v2/paged_kv_write.cu:72-81)
//   gather out[t][h][d] = K[(blocks[t / bs] * H + h) * bs + t % bs][d]
//          (KVFlux src/v2/paged_kv_read.cu:77-85)
#include <algorithm>

#include "common.cuh"
#include "launch.h"

namespace kvfx {
namespace {

template <int VB> struct Vec;
template <> struct Vec<16> { using T = uint4; };
template <> struct Vec<8> { using T = uint2; };
template <> struct Vec<4> { using T = uint32_t; };
template <> struct Vec<2> { using T = uint16_t; };
template <> struct Vec<1> { using T = uint8_t; };

// ------------------------------------------------------------------ write ---
// Thread i moves vector c of row (token, head) for both K and V; consecutive
// threads cover consecutive vectors of a row, so a 256-byte row is one fully
// coalesced 256-byte read and one 256-byte write.
template <int VB, typename Idx>
__global__ void __launch_bounds__(256) write_kernel(
    const typename Vec<VB>::T* __restrict__ k_new, const typename Vec<VB>::T* __restrict__ v_new,
    const uint64_t* __restrict__ slots, typename Vec<VB>::T* __restrict__ k_cache,
    typename Vec<VB>::T* __restrict__ v_cache, Idx total, Idx heads, Idx vpr, Idx bs,
    uint64_t slot_count, unsigned* status) {
    const Idx stride = static_cast<Idx>(gridDim.x) * blockDim.x;
    for (Idx i = static_cast<Idx>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
        const Idx row = i / vpr;
        const Idx c = i - row * vpr;
        const Idx tok = row / heads;
        const Idx h = row - tok * heads;
        const uint64_t slot = __ldg(slots + tok);
        if (slot >= slot_count) {
            raise_flag(status, KVFX_FLAG_BAD_INDEX);
            continue;
        }
        const uint64_t page = slot / bs;
        const uint64_t off = slot - page * bs;
        const uint64_t dst = ((page * heads + h) * bs + off) * vpr + c;
        const auto kv = __ldg(k_new + i);
        const auto vv = __ldg(v_new + i);
        k_cache[dst] = kv;
        v_cache[dst] = vv;
    }
}

template <int VB>
cudaError_t write_vb(const CacheView& c, const void* k_new, const void* v_new, const uint64_t* slots,
                     uint64_t n, unsigned* status, cudaStream_t s) {
    using V = typename Vec<VB>::T;
    const uint64_t vpr = c.row_bytes / VB;
    const uint64_t total = n * c.heads * vpr;
    const uint64_t want = ceil_div(total, 256);
    const uint32_t grid = static_cast<uint32_t>(std::min<uint64_t>(want, 148ull * 64));
    if (total < (1ull << 31)) {
        write_kernel<VB, uint32_t><<<grid, 256, 0, s>>>(
            static_cast<const V*>(k_new), static_cast<const V*>(v_new), slots, reinterpret_cast<V*>(c.k),
            reinterpret_cast<V*>(c.v), static_cast<uint32_t>(total), c.heads,
            static_cast<uint32_t>(vpr), c.bs, c.slot_count, status);
    } else {
        write_kernel<VB, uint64_t><<<grid, 256, 0, s>>>(
            static_cast<const V*>(k_new), static_cast<const V*>(v_new), slots, reinterpret_cast<V*>(c.k),
            reinterpret_cast<V*>(c.v), total, c.heads, vpr, c.bs, c.slot_count, status);
    }
    return cudaGetLastError();
}

// -------------------------------------------------------------- page copy ---
template <int VB>
__global__ void __launch_bounds__(256) copy_page_kernel(const typename Vec<VB>::T* __restrict__ ks,
                                                        const typename Vec<VB>::T* __restrict__ vs,
                                                        typename Vec<VB>::T* __restrict__ kd,
                                                        typename Vec<VB>::T* __restrict__ vd,
                                                        uint32_t n) {
    const uint32_t stride = gridDim.x * blockDim.x;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        kd[i] = ks[i];
        vd[i] = vs[i];
    }
}

template <int VB>
cudaError_t copy_vb(const CacheView& c, uint64_t src, uint64_t dst, cudaStream_t s) {
    using V = typename Vec<VB>::T;
    const uint64_t n = c.page_bytes / VB;
    const uint32_t grid = static_cast<uint32_t>(std::min<uint64_t>(ceil_div(n, 256), 1024));
    copy_page_kernel<VB><<<grid, 256, 0, s>>>(
        reinterpret_cast<const V*>(c.k + src * c.page_bytes),
        reinterpret_cast<const V*>(c.v + src * c.page_bytes),
        reinterpret_cast<V*>(c.k + dst * c.page_bytes), reinterpret_cast<V*>(c.v + dst * c.page_bytes),
        static_cast<uint32_t>(n));
    return cudaGetLastError();
}

// ------------------------------------------------------------ gather (SIMT) ---
// Generic gather for any row width: blockIdx.y selects the sequence, the x
// dimension strides over its (token, head, vector) elements.
template <int VB>
__global__ void __launch_bounds__(256) gather_simt_kernel(
    const typename Vec<VB>::T* __restrict__ k_cache, const typename Vec<VB>::T* __restrict__ v_cache,
    const uint64_t* __restrict__ blocks, uint64_t max_blocks, const uint64_t* __restrict__ lens,
    uint64_t single_len, void* const* k_list, void* const* v_list, void* k_one, void* v_one,
    uint32_t heads, uint32_t bs, uint32_t vpr, uint64_t num_blocks, unsigned* status) {
    using V = typename Vec<VB>::T;
    const uint64_t b = blockIdx.y;
    const uint64_t len = lens != nullptr ? lens[b] : single_len;
    const uint64_t* row_blocks = blocks + b * max_blocks;
    V* k_out = static_cast<V*>(k_list != nullptr ? k_list[b] : k_one);
    V* v_out = static_cast<V*>(v_list != nullptr ? v_list[b] : v_one);
    if (((reinterpret_cast<uintptr_t>(k_out) | reinterpret_cast<uintptr_t>(v_out)) % VB) != 0) {
        // Batched outputs are only known on the device: refuse a misaligned one.
        if (threadIdx.x == 0 && blockIdx.x == 0) raise_flag(status, KVFX_FLAG_BAD_INDEX);
        return;
    }
    if (ceil_div(len, bs) > max_blocks) {  // length beyond the table row
        if (threadIdx.x == 0 && blockIdx.x == 0) raise_flag(status, KVFX_FLAG_BAD_INDEX);
        return;
    }
    const uint64_t total = len * heads * vpr;
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += stride) {
        const uint64_t row = i / vpr;
        const uint64_t cc = i - row * vpr;
        const uint64_t t = row / heads;
        const uint64_t h = row - t * heads;
        const uint64_t lb = t / bs;
        const uint64_t blk = __ldg(row_blocks + lb);
        if (blk >= num_blocks) {
            raise_flag(status, KVFX_FLAG_BAD_INDEX);
            continue;
        }
        const uint64_t src = ((blk * heads + h) * bs + (t - lb * bs)) * vpr + cc;
        const V kv = __ldg(k_cache + src);
        const V vv = __ldg(v_cache + src);
        k_out[i] = kv;
        v_out[i] = vv;
    }
}

template <int VB>
cudaError_t gather_simt_vb(const CacheView& c, const GatherArgs& a, unsigned* status, cudaStream_t s) {
    using V = typename Vec<VB>::T;
    const uint64_t vpr = c.row_bytes / VB;
    const uint64_t per_seq = a.max_len * c.heads * vpr;
    const uint64_t seq_blocks = std::max<uint64_t>(1, (148ull * 16) / std::max<uint64_t>(1, a.batch));
    const uint32_t gx = static_cast<uint32_t>(std::min<uint64_t>(ceil_div(per_seq, 256), seq_blocks));
    dim3 grid(std::max<uint32_t>(gx, 1), static_cast<uint32_t>(a.batch));
    gather_simt_kernel<VB><<<grid, 256, 0, s>>>(
        reinterpret_cast<const V*>(c.k), reinterpret_cast<const V*>(c.v), a.blocks, a.max_blocks,
        a.lens, a.single_len, a.k_out_list, a.v_out_list, a.k_out, a.v_out, c.heads, c.bs,
        static_cast<uint32_t>(vpr), c.num_blocks, status);
    return cudaGetLastError();
}

// ------------------------------------------------------------- gather (TMA) ---
// Unit = one head of one page: a contiguous chunk [bs][head_size] in K and in
// V. One warp per CTA runs an S-stage ring: lane 0 brings a unit's K and V
// chunks into shared memory with two bulk (TMA) loads that complete on the
// stage's mbarrier; then the 32 lanes write the chunk's rows out with 16-byte
// stores (row t of the chunk is token j*bs+t, head h, of the output; a row is
// written by consecutive lanes, so each row is one coalesced run), and lane 0
// refills the stage with the unit S iterations ahead.
constexpr int kGatherMaxStages = 8;
constexpr int kGatherCtasPerSm = 6;

__global__ void __launch_bounds__(32) gather_tma_kernel(
    const char* __restrict__ k_cache, const char* __restrict__ v_cache,
    const uint64_t* __restrict__ blocks, uint64_t max_blocks, const uint64_t* __restrict__ lens,
    uint64_t single_len, void* const* k_list, void* const* v_list, void* k_one, void* v_one,
    uint32_t heads, uint32_t bs, uint32_t row_bytes, uint32_t chunk_bytes, uint32_t stages,
    uint64_t num_blocks, unsigned* status) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ uint64_t full[kGatherMaxStages];

    const uint32_t lane = threadIdx.x;
    const uint64_t b = blockIdx.y;
    const uint64_t len = lens != nullptr ? lens[b] : single_len;
    if (len == 0) return;
    const uint64_t* row_blocks = blocks + b * max_blocks;
    char* k_out = static_cast<char*>(k_list != nullptr ? k_list[b] : k_one);
    char* v_out = static_cast<char*>(v_list != nullptr ? v_list[b] : v_one);
    if (((reinterpret_cast<uintptr_t>(k_out) | reinterpret_cast<uintptr_t>(v_out)) & 15u) != 0) {
        // 16-byte stores need 16-byte aligned outputs (batched ones are only known here).
        if (lane == 0 && blockIdx.x == 0) raise_flag(status, KVFX_FLAG_BAD_INDEX);
        return;
    }
    const uint64_t pages = ceil_div(len, bs);
    if (pages > max_blocks) {  // length beyond the table row
        if (lane == 0 && blockIdx.x == 0) raise_flag(status, KVFX_FLAG_BAD_INDEX);
        return;
    }
    const uint64_t units = pages * heads;
    const uint64_t first = blockIdx.x;
    const uint64_t step = gridDim.x;
    if (first >= units) return;
    const uint32_t vpr = row_bytes / 16;  // 16-byte vectors per row

    if (lane == 0) {
        for (uint32_t st = 0; st < stages; ++st) mbar_init(&full[st], 1);
        fence_mbarrier_init();
    }
    __syncwarp();

    // Lane 0: start the loads of iteration `it` into stage it % stages.
    auto issue = [&](uint64_t it) {
        const uint64_t u = first + it * step;
        if (u >= units) return;
        const uint64_t j = u / heads;
        const uint64_t h = u - j * heads;
        uint64_t blk = __ldg(row_blocks + j);
        if (blk >= num_blocks) {
            raise_flag(status, KVFX_FLAG_BAD_INDEX);
            blk = 0;  // read something inside the cache; the flag reports the fault
        }
        const uint64_t off = (blk * heads + h) * static_cast<uint64_t>(chunk_bytes);
        const uint32_t st = static_cast<uint32_t>(it % stages);
        unsigned char* sk = smem + static_cast<size_t>(2 * st) * chunk_bytes;
        mbar_arrive_expect_tx(&full[st], 2 * chunk_bytes);
        bulk_g2s(sk, k_cache + off, chunk_bytes, &full[st]);
        bulk_g2s(sk + chunk_bytes, v_cache + off, chunk_bytes, &full[st]);
    };

    if (lane == 0) {
        for (uint32_t it = 0; it < stages; ++it) issue(it);
    }
    const uint64_t my_iters = ceil_div(units - first, step);
    for (uint64_t it = 0; it < my_iters; ++it) {
        const uint32_t st = static_cast<uint32_t>(it % stages);
        const uint32_t phase = static_cast<uint32_t>((it / stages) & 1);
        if (!mbar_wait(&full[st], phase, status)) break;  // flagged; stop issuing
        const uint64_t u = first + it * step;
        const uint64_t j = u / heads;
        const uint64_t h = u - j * heads;
        const uint64_t t0 = j * bs;
        const uint32_t rows = static_cast<uint32_t>(umin64(bs, len - t0));
        const uint4* sk = reinterpret_cast<const uint4*>(smem + static_cast<size_t>(2 * st) * chunk_bytes);
        const uint4* sv = sk + chunk_bytes / 16;
        const uint32_t n = rows * vpr;
        for (uint32_t i = lane; i < n; i += 32) {
            const uint32_t t = i / vpr;
            const uint32_t c = i - t * vpr;
            const uint64_t dst = ((t0 + t) * heads + h) * static_cast<uint64_t>(row_bytes) + c * 16u;
            const uint4 kx = sk[i];
            const uint4 vx = sv[i];
            __stcs(reinterpret_cast<uint4*>(k_out + dst), kx);
            __stcs(reinterpret_cast<uint4*>(v_out + dst), vx);
        }
        __syncwarp();  // every lane has read the stage
        if (lane == 0) {
            fence_proxy_async_smem();  // order those reads before the refill's async writes
            issue(it + stages);
        }
    }
}

}  // namespace

uint32_t vector_width(uint64_t bytes, const void* const* ptrs, int n) {
    for (uint32_t w : {16u, 8u, 4u, 2u}) {
        if (bytes % w != 0) continue;
        bool aligned = true;
        for (int i = 0; i < n; ++i) {
            if (reinterpret_cast<uintptr_t>(ptrs[i]) % w != 0) aligned = false;
        }
        if (aligned) return w;
    }
    return 1;
}

cudaError_t launch_write(const CacheView& c, const void* k_new, const void* v_new,
                         const uint64_t* slots, uint64_t n, unsigned* status, cudaStream_t s) {
    const void* ptrs[4] = {k_new, v_new, c.k, c.v};
    switch (vector_width(c.row_bytes, ptrs, 4)) {
    case 16: return write_vb<16>(c, k_new, v_new, slots, n, status, s);
    case 8: return write_vb<8>(c, k_new, v_new, slots, n, status, s);
    case 4: return write_vb<4>(c, k_new, v_new, slots, n, status, s);
    case 2: return write_vb<2>(c, k_new, v_new, slots, n, status, s);
    default: return write_vb<1>(c, k_new, v_new, slots, n, status, s);
    }
}

cudaError_t launch_copy_page(const CacheView& c, uint64_t src, uint64_t dst, unsigned*,
                             cudaStream_t s) {
    const void* ptrs[2] = {c.k, c.v};
    switch (vector_width(c.page_bytes, ptrs, 2)) {
    case 16: return copy_vb<16>(c, src, dst, s);
    case 8: return copy_vb<8>(c, src, dst, s);
    case 4: return copy_vb<4>(c, src, dst, s);
    case 2: return copy_vb<2>(c, src, dst, s);
    default: return copy_vb<1>(c, src, dst, s);
    }
}

cudaError_t launch_gather(const CacheView& c, const GatherArgs& a, unsigned* status, cudaStream_t s) {
    if (a.batch == 0 || a.max_len == 0) return cudaSuccess;
    // TMA path: rows must be whole 16-byte runs and both chunks of a stage fit.
    const bool single = a.k_out_list == nullptr;
    bool tma = c.row_bytes % 16 == 0 && c.chunk_bytes <= 32768 &&
               (reinterpret_cast<uintptr_t>(c.k) | reinterpret_cast<uintptr_t>(c.v)) % 16 == 0;
    if (tma && single) {
        tma = reinterpret_cast<uintptr_t>(a.k_out) % 16 == 0 &&
              reinterpret_cast<uintptr_t>(a.v_out) % 16 == 0;
    }
    // Batched outputs are checked on the device side only for 16-byte
    // alignment of the row size; the entry point verifies pointer alignment.
    if (tma) {
        const uint32_t stages = static_cast<uint32_t>(
            std::min<uint64_t>(kGatherMaxStages, std::max<uint64_t>(2, 32768 / (2 * c.chunk_bytes))));
        const size_t smem = static_cast<size_t>(stages) * 2 * c.chunk_bytes;
        static bool attr_set[64] = {false};  // the attribute is set once per device
        if (c.device < 0 || c.device >= 64 || !attr_set[c.device]) {
            cudaError_t e = cudaFuncSetAttribute(gather_tma_kernel,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, 131072);
            if (e != cudaSuccess) return e;
            if (c.device >= 0 && c.device < 64) attr_set[c.device] = true;
        }
        const uint64_t units_max = ceil_div(a.max_len, c.bs) * c.heads;
        const int sms = device_sm_count(c.device);
        const uint64_t ctas_total = static_cast<uint64_t>(sms) * kGatherCtasPerSm;
        const uint64_t per_seq = std::max<uint64_t>(1, ctas_total / a.batch);
        const uint32_t gx = static_cast<uint32_t>(std::min<uint64_t>(units_max, per_seq));
        dim3 grid(gx, static_cast<uint32_t>(a.batch));
        gather_tma_kernel<<<grid, 32, smem, s>>>(
            c.k, c.v, a.blocks, a.max_blocks, a.lens, a.single_len, a.k_out_list, a.v_out_list,
            a.k_out, a.v_out, c.heads, c.bs, static_cast<uint32_t>(c.row_bytes),
            static_cast<uint32_t>(c.chunk_bytes), stages, c.num_blocks, status);
        return cudaGetLastError();
    }
    const void* ptrs[4] = {c.k, c.v, single ? a.k_out : nullptr, single ? a.v_out : nullptr};
    switch (vector_width(c.row_bytes, ptrs, single ? 4 : 2)) {
    case 16: return gather_simt_vb<16>(c, a, status, s);
    case 8: return gather_simt_vb<8>(c, a, status, s);
    case 4: return gather_simt_vb<4>(c, a, status, s);
    case 2: return gather_simt_vb<2>(c, a, status, s);
    default: return gather_simt_vb<1>(c, a, status, s);
    }
}

}  // namespace kvfx
