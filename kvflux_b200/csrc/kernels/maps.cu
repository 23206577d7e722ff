// TMA tensor maps over a paged K/V cache, and small per-device facts.
//
// The decode kernel loads one 16-token tile of one KV head per page through a
// 4-D map {head_size, block_size, num_kv_heads, num_blocks} with a box of
// {64, 16, 1, 1} elements and the 128-byte swizzle (64 16-bit elements = one
// 128-byte swizzle span). Maps are encoded once per cache and kept for the
// life of the process (a few hundred bytes each).
#include <atomic>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "launch.h"

namespace kvfx {

namespace {

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                 CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                 CUtensorMapFloatOOBfill);

EncodeTiled encoder(cudaError_t* err) {
    static EncodeTiled fn = nullptr;
    static std::once_flag once;
    static cudaError_t status = cudaSuccess;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        status = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
        if (status == cudaSuccess && q == cudaDriverEntryPointSuccess) fn = reinterpret_cast<EncodeTiled>(p);
        else if (status == cudaSuccess) status = cudaErrorSymbolNotFound;
    });
    *err = status;
    return fn;
}

struct Entry {
    const void* k;
    const void* v;
    uint64_t num_blocks;
    uint32_t heads, bs, hd, dtype;
    CacheMaps* maps;
};

std::mutex g_mu;
std::vector<Entry> g_entries;

bool encode_one(EncodeTiled fn, CUtensorMap* map, void* base, const CacheView& c) {
    const CUtensorMapDataType t =
        c.dtype == KVFX_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const cuuint64_t dims[4] = {c.hd, c.bs, c.heads, c.num_blocks};
    const cuuint64_t strides[3] = {c.row_bytes, c.chunk_bytes, c.page_bytes};
    const cuuint32_t box[4] = {64, c.bs, 1, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    return fn(map, t, 4, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

const CacheMaps* cache_maps(const CacheView& c, cudaError_t* err) {
    *err = cudaSuccess;
    std::lock_guard<std::mutex> lock(g_mu);
    for (const Entry& e : g_entries) {
        if (e.k == c.k && e.v == c.v && e.num_blocks == c.num_blocks && e.heads == c.heads &&
            e.bs == c.bs && e.hd == c.hd && e.dtype == c.dtype) {
            return e.maps;
        }
    }
    EncodeTiled fn = encoder(err);
    if (fn == nullptr) return nullptr;
    CacheMaps* m = new CacheMaps();
    m->valid = encode_one(fn, &m->k, c.k, c) && encode_one(fn, &m->v, c.v, c);
    if (!m->valid) {
        delete m;
        *err = cudaErrorInvalidValue;
        return nullptr;
    }
    // A cache freed and re-allocated at the same address with the same shape
    // reuses the entry: the map only encodes address and shape.
    g_entries.push_back({c.k, c.v, c.num_blocks, c.heads, c.bs, c.hd, c.dtype, m});
    return m;
}

bool encode_tiled(CUtensorMap* map, CUtensorMapDataType type, uint32_t rank, void* base, const uint64_t* dims,
                  const uint64_t* strides, const uint32_t* box, cudaError_t* err) {
    *err = cudaSuccess;
    EncodeTiled fn = encoder(err);
    if (fn == nullptr) return false;
    cuuint64_t d[5], st[4];
    cuuint32_t b[5], e[5];
    for (uint32_t i = 0; i < rank; ++i) {
        d[i] = dims[i];
        b[i] = box[i];
        e[i] = 1;
        if (i + 1 < rank) st[i] = strides[i];
    }
    const bool ok = fn(map, type, rank, base, d, st, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                       CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    if (!ok) *err = cudaErrorInvalidValue;
    return ok;
}

namespace {

struct GatherEntry {
    const void* k;
    const void* v;
    uint64_t num_blocks;
    uint32_t heads, bs, hd, elem;
    CacheMaps* maps;
};
std::mutex g_gather_mu;
std::vector<GatherEntry> g_gather_entries;

}  // namespace

const CacheMaps* gather_maps(const CacheView& c, cudaError_t* err) {
    *err = cudaSuccess;
    std::lock_guard<std::mutex> lock(g_gather_mu);
    for (const GatherEntry& e : g_gather_entries) {
        if (e.k == c.k && e.v == c.v && e.num_blocks == c.num_blocks && e.heads == c.heads && e.bs == c.bs &&
            e.hd == c.hd && e.elem == c.elem) {
            return e.maps;
        }
    }
    // [num_blocks][heads][bs][hd] as a 4-D tensor of 2- or 4-byte elements;
    // one box = one (page, head) tile of bs rows, unswizzled.
    const CUtensorMapDataType t = c.elem == 4 ? CU_TENSOR_MAP_DATA_TYPE_UINT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16;
    const uint64_t dims[4] = {c.hd, c.bs, c.heads, c.num_blocks};
    const uint64_t strides[3] = {c.row_bytes, c.chunk_bytes, c.page_bytes};
    const uint32_t box[4] = {c.hd, c.bs, 1, 1};
    CacheMaps* m = new CacheMaps();
    m->valid = encode_tiled(&m->k, t, 4, c.k, dims, strides, box, err) &&
               encode_tiled(&m->v, t, 4, c.v, dims, strides, box, err);
    if (!m->valid) {
        delete m;
        return nullptr;
    }
    g_gather_entries.push_back({c.k, c.v, c.num_blocks, c.heads, c.bs, c.hd, c.elem, m});
    return m;
}

int device_sm_count(int device) {
    static std::atomic<int> counts[64];  // zero-initialised (static storage)
    if (device < 0 || device >= 64) return 148;
    int n = counts[device].load(std::memory_order_relaxed);
    if (n == 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0) {
            (void)cudaGetLastError();
            n = 148;
        }
        counts[device].store(n, std::memory_order_relaxed);
    }
    return n;
}

}  // namespace kvfx
