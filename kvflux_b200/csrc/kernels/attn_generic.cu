// Generic PagedAttention on CUDA cores, FP32 accumulation.
//
// Covers every shape the specialised kernels do not: FP32 caches, head sizes
// that are not a multiple of 64 (the reference's tests use 1..4 and 32),
// block sizes other than 16, GQA groups above 8. One warp owns one query row
// (query token or request, Q head): lanes take 32 tokens at a time for the
// scores, the chunk's softmax update is a warp reduction, and for the
// weighted sum lane l owns output dimensions l, l+32, ...
//
// Semantics follow the reference (KVFlux src/v2/paged_attention.cu:74-153):
// KV head = q_head / (q_heads / kv_heads); a single sequence's query i sees
// positions <= kv_tokens - query_tokens + i; a batch row sees all
// sequence_lengths[r] positions.
#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "launch.h"

namespace kvfx {
namespace {

constexpr int kWarps = 4;

struct GenericParams {
    const float* q;
    float* o;
    const char* k_cache;
    const char* v_cache;
    const uint64_t* blocks;
    uint64_t row_stride;
    const uint64_t* lens;
    uint64_t units;
    uint64_t kv_tokens;
    uint64_t num_blocks;
    uint32_t q_heads, kv_heads, bs, hd;
    float qscale;
    unsigned* status;
};

template <typename T, int NV>
__global__ void __launch_bounds__(kWarps * 32) attn_generic_kernel(const GenericParams p) {
    extern __shared__ float q_s[];  // [kWarps][hd]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint64_t row_id = static_cast<uint64_t>(blockIdx.x) * kWarps + warp;
    if (row_id >= p.units * p.q_heads) return;
    const uint64_t u = row_id / p.q_heads;
    const uint32_t qh = static_cast<uint32_t>(row_id - u * p.q_heads);
    const uint32_t kh = qh / (p.q_heads / p.kv_heads);

    uint64_t visible;
    const uint64_t* brow;
    if (p.lens != nullptr) {
        visible = p.lens[u];
        brow = p.blocks + u * p.row_stride;
        if (visible == 0 || visible > p.row_stride * p.bs) {  // outside the table row: refuse
            if (lane == 0) raise_flag(p.status, KVFX_FLAG_BAD_INDEX);
            return;
        }
    } else {
        visible = p.kv_tokens - p.units + u + 1;
        brow = p.blocks;
    }
    const T* kc = reinterpret_cast<const T*>(p.k_cache);
    const T* vc = reinterpret_cast<const T*>(p.v_cache);

    float* qv = q_s + warp * p.hd;
    const float* qsrc = p.q + row_id * p.hd;
    for (uint32_t d = lane; d < p.hd; d += 32) qv[d] = qsrc[d] * p.qscale;
    __syncwarp();

    float m = -INFINITY, l = 0.f;
    float acc[NV];
#pragma unroll
    for (int v = 0; v < NV; ++v) acc[v] = 0.f;

    for (uint64_t base = 0; base < visible; base += 32) {
        const uint64_t t = base + lane;
        float s = -INFINITY;
        uint64_t rowoff = 0;
        if (t < visible) {
            const uint64_t lb = t / p.bs;
            uint64_t blk = __ldg(brow + lb);
            if (blk >= p.num_blocks) {
                raise_flag(p.status, KVFX_FLAG_BAD_INDEX);
                blk = 0;
            }
            rowoff = ((blk * p.kv_heads + kh) * p.bs + (t - lb * p.bs)) * p.hd;
            const T* kr = kc + rowoff;
            float dot = 0.f;
            for (uint32_t d = 0; d < p.hd; ++d) dot = fmaf(qv[d], Elem<T>::to_f32(kr[d]), dot);
            s = dot;
        }
        float cm = s;
#pragma unroll
        for (int x = 16; x > 0; x >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, x));
        const float m_new = fmaxf(m, cm);
        const float alpha = exp2f(m - m_new);
        const float pw = exp2f(s - m_new);
        float ps = pw;
#pragma unroll
        for (int x = 16; x > 0; x >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, x);
        l = l * alpha + ps;
#pragma unroll
        for (int v = 0; v < NV; ++v) acc[v] *= alpha;
        const int n = static_cast<int>(umin64(32, visible - base));
        for (int jj = 0; jj < n; ++jj) {
            const float pj = __shfl_sync(0xffffffffu, pw, jj);
            const uint64_t offj = __shfl_sync(0xffffffffu, rowoff, jj);
            const T* vr = vc + offj;
#pragma unroll
            for (int v = 0; v < NV; ++v) {
                const uint32_t d = lane + 32u * v;
                if (d < p.hd) acc[v] = fmaf(pj, Elem<T>::to_f32(vr[d]), acc[v]);
            }
        }
        m = m_new;
    }
    const float inv = 1.f / l;
    float* out = p.o + row_id * p.hd;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
        const uint32_t d = lane + 32u * v;
        if (d < p.hd) out[d] = acc[v] * inv;
    }
}

template <typename T, int NV>
cudaError_t launch_nv(const GenericParams& p, cudaStream_t s) {
    const uint64_t rows = p.units * p.q_heads;
    const uint64_t grid = ceil_div(rows, kWarps);
    const size_t smem = static_cast<size_t>(kWarps) * p.hd * sizeof(float);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(attn_generic_kernel<T, NV>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    attn_generic_kernel<T, NV><<<static_cast<unsigned>(grid), kWarps * 32, smem, s>>>(p);
    return cudaGetLastError();
}

template <typename T>
cudaError_t launch_t(const GenericParams& p, cudaStream_t s) {
    if (p.hd <= 32) return launch_nv<T, 1>(p, s);
    if (p.hd <= 64) return launch_nv<T, 2>(p, s);
    if (p.hd <= 128) return launch_nv<T, 4>(p, s);
    if (p.hd <= 256) return launch_nv<T, 8>(p, s);
    if (p.hd <= 512) return launch_nv<T, 16>(p, s);
    return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t launch_attention_generic(const CacheView& c, const GenericAttnArgs& a, unsigned* status,
                                     cudaStream_t s) {
    if (a.units == 0) return cudaSuccess;
    GenericParams p;
    p.q = a.q;
    p.o = a.o;
    p.k_cache = c.k;
    p.v_cache = c.v;
    p.blocks = a.blocks;
    p.row_stride = a.row_stride;
    p.lens = a.lens;
    p.units = a.units;
    p.kv_tokens = a.kv_tokens;
    p.num_blocks = c.num_blocks;
    p.q_heads = a.q_heads;
    p.kv_heads = c.heads;
    p.bs = c.bs;
    p.hd = c.hd;
    p.qscale = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(c.hd)));
    p.status = status;
    switch (c.dtype) {
    case KVFX_F16: return launch_t<__half>(p, s);
    case KVFX_BF16: return launch_t<__nv_bfloat16>(p, s);
    default: return launch_t<float>(p, s);
    }
}

}  // namespace kvfx
