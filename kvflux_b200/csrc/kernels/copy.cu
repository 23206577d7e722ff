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
#include <atomic>
#include <utility>

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
    pdl_allow_next();
    pdl_wait();  // launched as a dependent: the previous kernel's writes first
    const Idx stride = static_cast<Idx>(gridDim.x) * blockDim.x;
    for (Idx i = static_cast<Idx>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
        const Idx row = i / vpr;
        const Idx c = i - row * vpr;
        const Idx tok = row / heads;
        const Idx h = row - tok * heads;
        // The row's data and its slot are loaded together (neither depends
        // on the other), so the thread waits for one memory latency, not two.
        const auto kv = __ldg(k_new + i);
        const auto vv = __ldg(v_new + i);
        const uint64_t slot = __ldg(slots + tok);
        if (slot >= slot_count) {
            raise_flag(status, KVFX_FLAG_BAD_INDEX);
            continue;
        }
        const uint64_t page = slot / bs;
        const uint64_t off = slot - page * bs;
        const uint64_t dst = ((page * heads + h) * bs + off) * vpr + c;
        k_cache[dst] = kv;
        v_cache[dst] = vv;
    }
}

// Launches `kernel` as a programmatic dependent of the stream's previous
// kernel: its CTAs may be scheduled while that kernel drains (the kernel
// waits for it with pdl_wait before touching memory). Short write launches
// that follow one another - a serving loop's steps, a graph of them - then
// lose the launch gap between them.
template <typename... KArgs, typename... Args>
cudaError_t launch_dependent(void (*kernel)(KArgs...), dim3 grid, dim3 block, cudaStream_t s, Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
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
        return launch_dependent(write_kernel<VB, uint32_t>, dim3(grid), dim3(256), s, static_cast<const V*>(k_new),
                                static_cast<const V*>(v_new), slots, reinterpret_cast<V*>(c.k),
                                reinterpret_cast<V*>(c.v), static_cast<uint32_t>(total),
                                static_cast<uint32_t>(c.heads), static_cast<uint32_t>(vpr),
                                static_cast<uint32_t>(c.bs), c.slot_count, status);
    }
    return launch_dependent(write_kernel<VB, uint64_t>, dim3(grid), dim3(256), s, static_cast<const V*>(k_new),
                            static_cast<const V*>(v_new), slots, reinterpret_cast<V*>(c.k), reinterpret_cast<V*>(c.v),
                            total, static_cast<uint64_t>(c.heads), vpr, static_cast<uint64_t>(c.bs), c.slot_count,
                            status);
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
    uint64_t single_len, void* const* k_list, void* const* v_list, void* k_one, void* v_one, uint64_t out_offset,
    uint32_t heads, uint32_t bs, uint32_t vpr, uint64_t num_blocks, unsigned* status) {
    using V = typename Vec<VB>::T;
    const uint64_t b = blockIdx.y;
    const uint64_t len = lens != nullptr ? lens[b] : single_len;
    const uint64_t* row_blocks = blocks + b * max_blocks;
    V* k_out = reinterpret_cast<V*>(static_cast<char*>(k_list != nullptr ? k_list[b] : k_one) + out_offset);
    V* v_out = reinterpret_cast<V*>(static_cast<char*>(v_list != nullptr ? v_list[b] : v_one) + out_offset);
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
        a.lens, a.single_len, a.k_out_list, a.v_out_list, a.k_out, a.v_out, a.out_offset, c.heads, c.bs,
        static_cast<uint32_t>(vpr), c.num_blocks, status);
    return cudaGetLastError();
}

// -------------------------------------------------------- gather (direct) ---
// Unit = one page of K and V: the contiguous [heads][bs][head_size] blocks go
// to contiguous [bs][heads][head_size] runs of the outputs. Each thread takes
// output vectors e = tid, tid + 256, ... in output order, so that a warp's
// stores are one 512-byte run and its loads two 256-byte rows; it holds
// kGatherDirectPer vectors of K and of V in flight before it stores any.
// One CTA per page (blockIdx.x; the loop covers grids capped below the page
// count) balances the tail across SMs best: measured on B200 at config 2,
// 1.02 of the plain device copy rate against 0.97 for 16 CTAs per SM and 0.84
// for a per-head TMA ring.
constexpr int kGatherDirectThreads = 256;
constexpr int kGatherDirectPer = 8;

// One page of one sequence: n output vectors (tokens of the page x heads x
// row vectors) from the page's K/V blocks ks/vs to the runs kd/vd; the same
// loop as gather_direct_kernel's (kept written out there: as a call it costs
// that kernel 16 registers and a CTA per SM).
__device__ __forceinline__ void gather_page(const uint4* ks, const uint4* vs,
                                            uint4* kd, uint4* vd, uint32_t n,
                                            uint32_t bs, uint32_t vpr, uint32_t vpt, FastDiv div_vpt,
                                            FastDiv div_vpr, uint32_t tid) {
    for (uint32_t base = 0; base < n; base += kGatherDirectThreads * kGatherDirectPer) {
        uint4 kx[kGatherDirectPer], vx[kGatherDirectPer];
#pragma unroll
        for (int i = 0; i < kGatherDirectPer; ++i) {
            const uint32_t e = base + i * kGatherDirectThreads + tid;
            if (e < n) {
                const uint32_t t = fast_div(e, div_vpt);
                const uint32_t r = e - t * vpt;
                const uint32_t h = fast_div(r, div_vpr);
                const uint32_t src = (h * bs + t) * vpr + (r - h * vpr);
                kx[i] = __ldg(ks + src);
                vx[i] = __ldg(vs + src);
            }
        }
#pragma unroll
        for (int i = 0; i < kGatherDirectPer; ++i) {
            const uint32_t e = base + i * kGatherDirectThreads + tid;
            if (e < n) {
                __stcs(kd + e, kx[i]);
                __stcs(vd + e, vx[i]);
            }
        }
    }
}

__global__ void __launch_bounds__(kGatherDirectThreads) gather_direct_kernel(
    const uint4* __restrict__ k_cache, const uint4* __restrict__ v_cache,
    const uint64_t* __restrict__ blocks, uint64_t max_blocks, const uint64_t* __restrict__ lens,
    uint64_t single_len, void* const* k_list, void* const* v_list, void* k_one, void* v_one,
    uint32_t heads, uint32_t bs, uint32_t vpr, FastDiv div_vpt, FastDiv div_vpr, uint64_t num_blocks,
    unsigned* status) {
    const uint32_t tid = threadIdx.x;
    const uint64_t b = blockIdx.y;
    const uint64_t len = lens != nullptr ? lens[b] : single_len;
    if (len == 0) return;
    const uint64_t* row_blocks = blocks + b * max_blocks;
    uint4* k_out = static_cast<uint4*>(k_list != nullptr ? k_list[b] : k_one);
    uint4* v_out = static_cast<uint4*>(v_list != nullptr ? v_list[b] : v_one);
    if (((reinterpret_cast<uintptr_t>(k_out) | reinterpret_cast<uintptr_t>(v_out)) & 15u) != 0) {
        if (tid == 0 && blockIdx.x == 0) raise_flag(status, KVFX_FLAG_BAD_INDEX);
        return;
    }
    const uint64_t pages = ceil_div(len, bs);
    if (pages > max_blocks) {
        if (tid == 0 && blockIdx.x == 0) raise_flag(status, KVFX_FLAG_BAD_INDEX);
        return;
    }
    const uint32_t vpt = heads * vpr;  // 16-byte vectors per token (all heads)
    const uint64_t page_vecs = static_cast<uint64_t>(bs) * vpt;
    for (uint64_t j = blockIdx.x; j < pages; j += gridDim.x) {
        const uint64_t blk = __ldg(row_blocks + j);
        if (blk >= num_blocks) {
            if (tid == 0) raise_flag(status, KVFX_FLAG_BAD_INDEX);
            continue;
        }
        const uint64_t t0 = j * bs;
        const uint32_t n = static_cast<uint32_t>(umin64(bs, len - t0)) * vpt;
        const uint4* ks = k_cache + blk * page_vecs;
        const uint4* vs = v_cache + blk * page_vecs;
        uint4* kd = k_out + t0 * vpt;
        uint4* vd = v_out + t0 * vpt;
        for (uint32_t base = 0; base < n; base += kGatherDirectThreads * kGatherDirectPer) {
            uint4 kx[kGatherDirectPer], vx[kGatherDirectPer];
#pragma unroll
            for (int i = 0; i < kGatherDirectPer; ++i) {
                const uint32_t e = base + i * kGatherDirectThreads + tid;
                if (e < n) {
                    const uint32_t t = fast_div(e, div_vpt);
                    const uint32_t r = e - t * vpt;
                    const uint32_t h = fast_div(r, div_vpr);
                    const uint32_t src = (h * bs + t) * vpr + (r - h * vpr);
                    kx[i] = __ldg(ks + src);
                    vx[i] = __ldg(vs + src);
                }
            }
#pragma unroll
            for (int i = 0; i < kGatherDirectPer; ++i) {
                const uint32_t e = base + i * kGatherDirectThreads + tid;
                if (e < n) {
                    __stcs(kd + e, kx[i]);
                    __stcs(vd + e, vx[i]);
                }
            }
        }
    }
}

// ---------------------------------------------------------- layer batches ---
// One launch over the caches of num_layers layers that share a page pool
// (one PagedKVStorage per layer): blockIdx.y (write) or blockIdx.z (gather)
// selects the layer, whose cache bases come from the kernel parameters.
struct LayerBases {
    char* k[KVFX_MAX_LAYERS];
    char* v[KVFX_MAX_LAYERS];
};

// Vectors of K and of V in flight per thread before its stores. Two (small
// CTAs, 38 registers, 6 CTAs per SM) measured faster than four or eight at
// config 2's 32-layer step (12.44 / 12.98 / 17.5 us per launch in a graph):
// finer CTAs even out the launch's last wave.
constexpr int kWriteLayersPer = 2;

__global__ void __launch_bounds__(256) write_layers_kernel(
    const __grid_constant__ LayerBases bases, const uint4* __restrict__ k_new, const uint4* __restrict__ v_new,
    uint64_t layer_stride_vecs, const uint64_t* __restrict__ slots, uint32_t total, uint32_t heads, uint32_t vpr,
    uint32_t bs, uint64_t slot_count, unsigned* status) {
    pdl_allow_next();
    pdl_wait();  // launched as a dependent: the previous kernel's writes first
    const uint32_t layer = blockIdx.y;
    const uint4* kn = k_new + layer * layer_stride_vecs;
    const uint4* vn = v_new + layer * layer_stride_vecs;
    uint4* kc = reinterpret_cast<uint4*>(bases.k[layer]);
    uint4* vc = reinterpret_cast<uint4*>(bases.v[layer]);
    // Each thread has kWriteLayersPer vectors of K and of V in flight before
    // it stores any (vector i = base + j * 256 + tid, in input order).
    const uint32_t span = gridDim.x * blockDim.x * kWriteLayersPer;
    for (uint32_t base = blockIdx.x * blockDim.x * kWriteLayersPer; base < total; base += span) {
        uint4 kx[kWriteLayersPer], vx[kWriteLayersPer];
        uint64_t dst[kWriteLayersPer];
        // Data and slots are loaded before any slot is examined: the data
        // loads do not depend on the slots, so both latencies overlap.
        uint64_t slot[kWriteLayersPer];
#pragma unroll
        for (int j = 0; j < kWriteLayersPer; ++j) {
            const uint32_t i = base + j * blockDim.x + threadIdx.x;
            slot[j] = ~0ull;
            if (i < total) {
                kx[j] = __ldg(kn + i);
                vx[j] = __ldg(vn + i);
                slot[j] = __ldg(slots + i / vpr / heads);
            }
        }
#pragma unroll
        for (int j = 0; j < kWriteLayersPer; ++j) {
            const uint32_t i = base + j * blockDim.x + threadIdx.x;
            dst[j] = ~0ull;
            if (i < total) {
                const uint32_t row = i / vpr;
                const uint32_t c = i - row * vpr;
                const uint32_t tok = row / heads;
                const uint32_t h = row - tok * heads;
                if (slot[j] < slot_count) {
                    const uint64_t page = slot[j] / bs;
                    const uint64_t off = slot[j] - page * bs;
                    dst[j] = ((page * heads + h) * bs + off) * vpr + c;
                } else {
                    raise_flag(status, KVFX_FLAG_BAD_INDEX);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < kWriteLayersPer; ++j) {
            if (dst[j] != ~0ull) {
                kc[dst[j]] = kx[j];
                vc[dst[j]] = vx[j];
            }
        }
    }
}

__global__ void __launch_bounds__(kGatherDirectThreads) gather_layers_kernel(
    const __grid_constant__ LayerBases bases, const uint64_t* __restrict__ blocks, uint64_t max_blocks,
    const uint64_t* __restrict__ lens, void* const* k_list, void* const* v_list, uint64_t out_layer_stride,
    uint32_t heads, uint32_t bs, uint32_t vpr, FastDiv div_vpt, FastDiv div_vpr, uint64_t num_blocks,
    unsigned* status) {
    const uint32_t tid = threadIdx.x;
    const uint64_t b = blockIdx.y;
    const uint32_t layer = blockIdx.z;
    const uint64_t len = lens[b];
    if (len == 0) return;
    const uint64_t* row_blocks = blocks + b * max_blocks;
    char* kb = static_cast<char*>(k_list[b]);
    char* vb = static_cast<char*>(v_list[b]);
    if (((reinterpret_cast<uintptr_t>(kb) | reinterpret_cast<uintptr_t>(vb)) & 15u) != 0) {
        if (tid == 0 && blockIdx.x == 0) raise_flag(status, KVFX_FLAG_BAD_INDEX);
        return;
    }
    uint4* k_out = reinterpret_cast<uint4*>(kb + layer * out_layer_stride);
    uint4* v_out = reinterpret_cast<uint4*>(vb + layer * out_layer_stride);
    const uint64_t pages = ceil_div(len, bs);
    if (pages > max_blocks) {
        if (tid == 0 && blockIdx.x == 0) raise_flag(status, KVFX_FLAG_BAD_INDEX);
        return;
    }
    const uint32_t vpt = heads * vpr;
    const uint64_t page_vecs = static_cast<uint64_t>(bs) * vpt;
    const uint4* k_cache = reinterpret_cast<const uint4*>(bases.k[layer]);
    const uint4* v_cache = reinterpret_cast<const uint4*>(bases.v[layer]);
    for (uint64_t j = blockIdx.x; j < pages; j += gridDim.x) {
        const uint64_t blk = __ldg(row_blocks + j);
        if (blk >= num_blocks) {
            if (tid == 0) raise_flag(status, KVFX_FLAG_BAD_INDEX);
            continue;
        }
        const uint64_t t0 = j * bs;
        const uint32_t n = static_cast<uint32_t>(umin64(bs, len - t0)) * vpt;
        gather_page(k_cache + blk * page_vecs, v_cache + blk * page_vecs, k_out + t0 * vpt, v_out + t0 * vpt, n,
                    bs, vpr, vpt, div_vpt, div_vpr, tid);
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

cudaError_t launch_write_layers(const CacheView* layers, uint32_t num_layers, const void* k_new,
                                const void* v_new, uint64_t layer_stride, const uint64_t* slots, uint64_t n,
                                unsigned* status, cudaStream_t s) {
    const CacheView& c = layers[0];
    const uint64_t total = n * c.heads * (c.row_bytes / 16);
    bool vec16 = c.row_bytes % 16 == 0 && layer_stride % 16 == 0 && total < (1ull << 31) &&
                 ((reinterpret_cast<uintptr_t>(k_new) | reinterpret_cast<uintptr_t>(v_new)) & 15u) == 0;
    for (uint32_t l = 0; l < num_layers && vec16; ++l) {
        vec16 = ((reinterpret_cast<uintptr_t>(layers[l].k) | reinterpret_cast<uintptr_t>(layers[l].v)) & 15u) == 0;
    }
    if (!vec16) {  // odd rows or alignments: one launch per layer
        for (uint32_t l = 0; l < num_layers; ++l) {
            const cudaError_t e = launch_write(layers[l], static_cast<const char*>(k_new) + l * layer_stride,
                                               static_cast<const char*>(v_new) + l * layer_stride, slots, n,
                                               status, s);
            if (e != cudaSuccess) return e;
        }
        return cudaSuccess;
    }
    LayerBases bases{};
    for (uint32_t l = 0; l < num_layers; ++l) {
        bases.k[l] = layers[l].k;
        bases.v[l] = layers[l].v;
    }
    const uint32_t gx = static_cast<uint32_t>(std::max<uint64_t>(
        1, std::min<uint64_t>(ceil_div(total, 256 * kWriteLayersPer), ceil_div(148ull * 16, num_layers))));
    return launch_dependent(write_layers_kernel, dim3(gx, num_layers), dim3(256), s, bases,
                            static_cast<const uint4*>(k_new), static_cast<const uint4*>(v_new), layer_stride / 16,
                            slots, static_cast<uint32_t>(total), static_cast<uint32_t>(c.heads),
                            static_cast<uint32_t>(c.row_bytes / 16), static_cast<uint32_t>(c.bs), c.slot_count,
                            status);
}

cudaError_t launch_gather_layers(const CacheView* layers, uint32_t num_layers, const GatherArgs& a,
                                 uint64_t out_layer_stride, unsigned* status, cudaStream_t s) {
    if (a.batch == 0 || a.max_len == 0) return cudaSuccess;
    const CacheView& c = layers[0];
    bool direct = c.row_bytes % 16 == 0 && c.page_bytes / 16 < (1ull << 31) && out_layer_stride % 16 == 0;
    for (uint32_t l = 0; l < num_layers && direct; ++l) {
        direct = ((reinterpret_cast<uintptr_t>(layers[l].k) | reinterpret_cast<uintptr_t>(layers[l].v)) & 15u) == 0;
    }
    if (!direct) return cudaErrorNotSupported;  // the C ABI routes these shapes per layer
    LayerBases bases{};
    for (uint32_t l = 0; l < num_layers; ++l) {
        bases.k[l] = layers[l].k;
        bases.v[l] = layers[l].v;
    }
    const uint32_t vpr = static_cast<uint32_t>(c.row_bytes / 16);
    const uint64_t pages_max = ceil_div(a.max_len, c.bs);
    dim3 grid(static_cast<uint32_t>(std::min<uint64_t>(pages_max, 0x7fffffffu)), static_cast<uint32_t>(a.batch),
              num_layers);
    gather_layers_kernel<<<grid, kGatherDirectThreads, 0, s>>>(
        bases, a.blocks, a.max_blocks, a.lens, a.k_out_list, a.v_out_list, out_layer_stride, c.heads, c.bs, vpr,
        make_fastdiv(c.heads * vpr), make_fastdiv(vpr), c.num_blocks, status);
    return cudaGetLastError();
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

// ------------------------------------------------------------- gather (TMA) ---
// One sequence gathered by the tensor memory accelerator. Unit = (page, KV
// head): its K and V tiles (block_size rows of head_size elements, one
// contiguous run in the cache) are loaded with one 4-D tensor copy each into
// shared memory and stored with one 3-D tensor copy each through maps over
// the outputs [tokens][heads][head_size] whose box is {head_size, 1 head,
// block_size tokens}: the box walks the heads' stride in global memory, so
// the page's [head][token] order becomes the output's [token][head] order
// with no work in shared memory. A store past the sequence's last token is
// clipped by the copy engine. One warp per CTA, one lane issuing: a ring of
// kGatherTmaSlots units; a slot is refilled once the stores that read it
// have finished reading (bulk-group waits). Tiles sit at 128-byte aligned
// shared-memory offsets (tile_stride), as tensor copies require.
constexpr int kGatherTmaSlots = 4;

__global__ void __launch_bounds__(32) gather_tma_kernel(
    const __grid_constant__ CUtensorMap in_k, const __grid_constant__ CUtensorMap in_v,
    const __grid_constant__ CUtensorMap out_k, const __grid_constant__ CUtensorMap out_v,
    const uint64_t* __restrict__ blocks, uint64_t num_tokens, uint32_t heads, uint32_t bs, uint32_t tile_bytes,
    uint32_t tile_stride, uint64_t num_blocks, unsigned* status) {
    extern __shared__ unsigned char smem_raw[];
    __shared__ uint64_t full[kGatherTmaSlots];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                           ~uintptr_t(1023));
    pdl_allow_next();
    if (!elect_one()) return;
    pdl_wait();  // launched as a dependent: the previous kernel's writes first
    const uint64_t pages = ceil_div(num_tokens, bs);
    const uint64_t units = pages * heads;
    const uint64_t first = blockIdx.x;
    const uint64_t n_my = first < units ? ceil_div(units - first, gridDim.x) : 0;
    for (int i = 0; i < kGatherTmaSlots; ++i) mbar_init(&full[i], 1);
    fence_mbarrier_init();
    prefetch_tensormap(&in_k);
    prefetch_tensormap(&in_v);
    prefetch_tensormap(&out_k);
    prefetch_tensormap(&out_v);
    bool skip[kGatherTmaSlots] = {};
    auto load = [&](uint64_t k) {  // unit k of this CTA into slot k % kGatherTmaSlots
        if (k >= n_my) return;
        const int st = static_cast<int>(k % kGatherTmaSlots);
        const uint64_t u = first + k * gridDim.x;
        const uint64_t page = u / heads;
        const uint32_t h = static_cast<uint32_t>(u - page * heads);
        const uint64_t blk = __ldg(blocks + page);
        skip[st] = blk >= num_blocks;
        if (skip[st]) {  // never followed: flagged, the output rows stay as they were
            raise_flag(status, KVFX_FLAG_BAD_INDEX);
            mbar_arrive(&full[st]);
            return;
        }
        unsigned char* dst = smem + st * 2 * tile_stride;
        mbar_arrive_expect_tx(&full[st], 2 * tile_bytes);
        tma_load_4d(dst, &in_k, 0, 0, static_cast<int>(h), static_cast<int>(blk), &full[st]);
        tma_load_4d(dst + tile_stride, &in_v, 0, 0, static_cast<int>(h), static_cast<int>(blk), &full[st]);
    };
    for (uint64_t k = 0; k + 1 < kGatherTmaSlots; ++k) load(k);
    uint64_t waited = 0;  // units whose loads this lane has seen complete
    for (uint64_t k = 0; k < n_my; ++k) {
        const int st = static_cast<int>(k % kGatherTmaSlots);
        if (!mbar_wait(&full[st], static_cast<uint32_t>(k / kGatherTmaSlots) & 1u, status)) break;
        waited = k + 1;
        if (!skip[st]) {
            fence_proxy_async_smem();
            const uint64_t u = first + k * gridDim.x;
            const uint64_t page = u / heads;
            const int h = static_cast<int>(u - page * heads);
            const int t0 = static_cast<int>(page * bs);
            const unsigned char* src = smem + st * 2 * tile_stride;
            tma_store_3d(&out_k, 0, h, t0, src);
            tma_store_3d(&out_v, 0, h, t0, src + tile_stride);
        }
        bulk_commit();
        bulk_wait_read<1>();  // unit k - 1's stores have read their slot
        load(k + kGatherTmaSlots - 1);
    }
    // Loads issued but not waited for (a wait gave up): let them land
    // (bounded) before the shared memory is released.
    const uint64_t issued = n_my < waited + kGatherTmaSlots - 1 ? n_my : waited + kGatherTmaSlots - 1;
    for (uint64_t k = waited; k < issued; ++k) {
        (void)mbar_wait(&full[k % kGatherTmaSlots], static_cast<uint32_t>(k / kGatherTmaSlots) & 1u, status);
    }
    bulk_wait<0>();
}

// One sequence through gather_tma_kernel, when its rows are whole 16-byte
// multiples of at most 256 elements, its tiles fit the ring (<= 8 KiB per
// tile) and every base is 16-byte aligned; false (nothing launched) otherwise.
bool gather_tma(const CacheView& c, const GatherArgs& a, unsigned* status, cudaStream_t s, cudaError_t* err) {
    *err = cudaSuccess;
    const uint64_t tile = static_cast<uint64_t>(c.bs) * c.row_bytes;
    if (c.row_bytes % 16 != 0 || c.hd > 256 || c.bs > 256 || tile > 8192 || a.single_len >= (1ull << 31) ||
        c.num_blocks >= (1ull << 31) || c.heads >= (1u << 31) || ((reinterpret_cast<uintptr_t>(c.k) |
        reinterpret_cast<uintptr_t>(c.v) | reinterpret_cast<uintptr_t>(a.k_out) |
        reinterpret_cast<uintptr_t>(a.v_out)) & 15u) != 0 || ceil_div(a.single_len, c.bs) > a.max_blocks) {
        return false;
    }
    const CacheMaps* in = gather_maps(c, err);
    if (in == nullptr) return false;
    const CUtensorMapDataType t = c.elem == 4 ? CU_TENSOR_MAP_DATA_TYPE_UINT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16;
    const uint64_t dims[3] = {c.hd, c.heads, a.single_len};
    const uint64_t strides[2] = {c.row_bytes, c.row_bytes * c.heads};
    const uint32_t box[3] = {c.hd, 1, c.bs};
    CUtensorMap out_k, out_v;
    if (!encode_tiled(&out_k, t, 3, a.k_out, dims, strides, box, err) ||
        !encode_tiled(&out_v, t, 3, a.v_out, dims, strides, box, err)) {
        return false;
    }
    const uint64_t tile_stride = (tile + 127) & ~uint64_t(127);  // tensor copies need 128-byte aligned smem
    const uint32_t smem = static_cast<uint32_t>(kGatherTmaSlots * 2 * tile_stride + 1024);
    static std::atomic<int> attr_done[64];
    if (c.device < 0 || c.device >= 64 || !attr_done[c.device].load(std::memory_order_acquire)) {
        *err = cudaFuncSetAttribute(gather_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 65536 + 1024);
        if (*err != cudaSuccess) return true;
        if (c.device >= 0 && c.device < 64) attr_done[c.device].store(1, std::memory_order_release);
    }
    const uint64_t units = ceil_div(a.single_len, c.bs) * c.heads;
    const uint64_t per_sm = std::max<uint64_t>(1, (227ull * 1024) / (smem + 1024));
    const uint32_t grid = static_cast<uint32_t>(std::min<uint64_t>(units, device_sm_count(c.device) * per_sm));
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    *err = cudaLaunchKernelEx(&cfg, gather_tma_kernel, in->k, in->v, out_k, out_v, a.blocks, a.single_len, c.heads,
                              c.bs, static_cast<uint32_t>(tile), static_cast<uint32_t>(tile_stride), c.num_blocks,
                              status);
    return true;
}

cudaError_t launch_gather(const CacheView& c, const GatherArgs& a, unsigned* status, cudaStream_t s) {
    if (a.batch == 0 || a.max_len == 0) return cudaSuccess;
    // Direct path: rows are whole 16-byte vectors, the caches and (for one
    // sequence) the outputs 16-byte aligned, and a page's vector indices fit
    // 31 bits. Batched outputs are only known on the device: the kernel
    // refuses a misaligned one with the bad-index flag.
    const bool single = a.k_out_list == nullptr;
    if (single && !a.force_simt && a.out_offset == 0 && a.single_len != 0) {
        cudaError_t e = cudaSuccess;
        if (gather_tma(c, a, status, s, &e)) return e;
    }
    bool direct = !a.force_simt && a.out_offset == 0 && c.row_bytes % 16 == 0 && c.page_bytes / 16 < (1ull << 31) &&
                  (reinterpret_cast<uintptr_t>(c.k) | reinterpret_cast<uintptr_t>(c.v)) % 16 == 0;
    if (direct && single) {
        direct = reinterpret_cast<uintptr_t>(a.k_out) % 16 == 0 && reinterpret_cast<uintptr_t>(a.v_out) % 16 == 0;
    }
    if (direct) {
        const uint32_t vpr = static_cast<uint32_t>(c.row_bytes / 16);
        const uint64_t pages_max = ceil_div(a.max_len, c.bs);
        const uint32_t gx = static_cast<uint32_t>(std::min<uint64_t>(pages_max, 0x7fffffffu));
        dim3 grid(gx, static_cast<uint32_t>(a.batch));
        gather_direct_kernel<<<grid, kGatherDirectThreads, 0, s>>>(
            reinterpret_cast<const uint4*>(c.k), reinterpret_cast<const uint4*>(c.v), a.blocks, a.max_blocks,
            a.lens, a.single_len, a.k_out_list, a.v_out_list, a.k_out, a.v_out, c.heads, c.bs, vpr,
            make_fastdiv(c.heads * vpr), make_fastdiv(vpr), c.num_blocks, status);
        return cudaGetLastError();
    }
    const void* ptrs[4] = {c.k, c.v, single ? a.k_out : nullptr, single ? a.v_out : nullptr};
    uint32_t width = vector_width(c.row_bytes, ptrs, single ? 4 : 2);
    while (width > 1 && a.out_offset % width != 0) width /= 2;
    switch (width) {
    case 16: return gather_simt_vb<16>(c, a, status, s);
    case 8: return gather_simt_vb<8>(c, a, status, s);
    case 4: return gather_simt_vb<4>(c, a, status, s);
    case 2: return gather_simt_vb<2>(c, a, status, s);
    default: return gather_simt_vb<1>(c, a, status, s);
    }
}

}  // namespace kvfx
