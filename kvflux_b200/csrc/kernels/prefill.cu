// Causal prefill PagedAttention on the 5th-generation tensor cores (kernel 4).
//
// One CTA = 128 query rows (a query tile) of one Q head of one sequence,
// against the KV tiles of 64 tokens (4 pages) that the tile's rows can see.
// Warp roles:
//   warp 0      TMA producer: per KV tile, 16 tensor loads (4 pages x 2
//               64-dim halves, K and V; 128-byte swizzle, no multicast) into a
//               3-stage ring.
//   warp 1      owns TMEM (256 columns: S0, S1, O) and issues every tcgen05.mma
//               from one thread: S_j = Q K_j^T into S[j%2] while the softmax
//               works on S[(j-1)%2], then O += P_{j-1} V_{j-1}.
//   warps 2..5  softmax, one query row per thread (TMEM lane = row): scores
//               from TMEM, causal mask, online softmax in base 2, P to shared
//               memory; at the end O / l from TMEM to global memory.
// Precision: Q (FP32 in the API) and P are each fed as two bf16/fp16
// operands, hi = round(x) and lo = round(x - hi), accumulated into the same
// TMEM tile (S = Q_hi K + Q_lo K, O += P_hi V + P_lo V), which keeps ~16
// mantissa bits and FP32-class error against the FP64 reference; rounding Q
// or P to 16 bits alone exceeds 2e-3 at 4096 tokens.
// O is rescaled in TMEM only when a tile's row maximum exceeds the running
// one by more than 8 (base-2 units). Tokens past the sequence end in the last
// tile are masked in S and zeroed in the V tile.
//
// Semantics: KVFlux src/v2/paged_attention.cu:109-128 (query i sees
// positions <= kv_tokens - query_tokens + i; KV head = q_head / group).
#include <cmath>
#include <type_traits>

#include "common.cuh"
#include "launch.h"
#include "tcgen05.cuh"

namespace kvfx {
namespace {

constexpr int kBM = 128;        // query rows per CTA
constexpr int kBN = 64;         // KV tokens per tile (4 pages of 16)
constexpr int kHD = 128;        // head size handled here
constexpr int kStages = 3;      // K/V ring depth
constexpr int kThreads = 192;   // 6 warps
constexpr uint32_t kTmemCols = 256;

// Shared-memory layout (byte offsets from a 1024-aligned base).
constexpr uint32_t kQAtom = kBM * 128;            // [128 rows][64 dims] 16-bit, 16 KiB
constexpr uint32_t kQBytes = 2 * kQAtom;          // 128 dims
constexpr uint32_t kKVHalf = kBN * 128;           // [64 tokens][64 dims], 8 KiB
constexpr uint32_t kKVTile = 2 * kKVHalf;         // 16 KiB
constexpr uint32_t kOffQHi = 0;
constexpr uint32_t kOffQLo = kOffQHi + kQBytes;
constexpr uint32_t kOffK = kOffQLo + kQBytes;
constexpr uint32_t kOffV = kOffK + kStages * kKVTile;
constexpr uint32_t kOffPHi = kOffV + kStages * kKVTile;
constexpr uint32_t kOffPLo = kOffPHi + kBM * 128;
constexpr uint32_t kSmemBytes = kOffPLo + kBM * 128;   // 192 KiB
constexpr uint32_t kSmemAlloc = kSmemBytes + 1024;

struct PrefillParams {
    const float* q;
    float* o;
    const uint64_t* blocks;
    uint64_t q_tokens, kv_tokens, num_blocks;
    uint32_t q_heads, kv_heads, group, n_qtiles;
    float qscale;
    unsigned* status;
};

// Byte offset of 16-byte chunk `c` of row `r` in a K-major 128-byte-swizzled
// atom of rows 128 bytes wide.
__device__ __forceinline__ uint32_t swz_row(uint32_t r, uint32_t c) {
    return (r >> 3) * 1024 + (r & 7) * 128 + (((c ^ r) & 7) << 4);
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
prefill_tc_kernel(const __grid_constant__ PrefillParams p, const __grid_constant__ CUtensorMap kmap,
                  const __grid_constant__ CUtensorMap vmap) {
    extern __shared__ unsigned char smem_raw[];
    __shared__ uint64_t kv_full[kStages], kv_empty[kStages];
    __shared__ uint64_t s_full[2], s_empty[2];
    __shared__ uint64_t q_full, p_full, o_done, mma_done;
    __shared__ uint32_t tmem_base_slot;
    __shared__ int abort_flag;

    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_addr(smem);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    const uint32_t qtile = p.n_qtiles - 1 - blockIdx.x;  // heaviest tiles first
    const uint32_t qh = blockIdx.y;
    const uint32_t kh = qh / p.group;
    const uint64_t q0 = static_cast<uint64_t>(qtile) * kBM;
    const uint64_t q_last = umin64(q0 + kBM, p.q_tokens) - 1;
    const uint64_t last_pos = p.kv_tokens - p.q_tokens + q_last;
    const uint32_t ntiles = static_cast<uint32_t>(last_pos / kBN + 1);
    const uint64_t npages = ceil_div(p.kv_tokens, 16);

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&s_full[s], 1);
            mbar_init(&s_empty[s], 128);
        }
        mbar_init(&q_full, 128);
        mbar_init(&p_full, 128);
        mbar_init(&o_done, 1);
        mbar_init(&mma_done, 1);
        abort_flag = 0;
        fence_mbarrier_init();
    }
    if (warp == 1) {
        tc::tmem_alloc(&tmem_base_slot, kTmemCols);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = tmem_base_slot;
    const uint32_t tS[2] = {tmem, tmem + kBN};
    const uint32_t tO = tmem + 2 * kBN;

    if (warp == 0) {
        // ------------------------------------------------------ producer ---
        if (lane == 0) {
            prefetch_tensormap(&kmap);
            prefetch_tensormap(&vmap);
            for (uint32_t j = 0; j < ntiles; ++j) {
                const int st = static_cast<int>(j % kStages);
                if (j >= kStages && !mbar_wait(&kv_empty[st], ((j - kStages) / kStages) & 1u, p.status)) {
                    abort_flag = 1;
                    break;
                }
                mbar_arrive_expect_tx(&kv_full[st], 2 * kKVTile);
                unsigned char* kt = smem + kOffK + st * kKVTile;
                unsigned char* vt = smem + kOffV + st * kKVTile;
#pragma unroll
                for (int pg = 0; pg < kBN / 16; ++pg) {
                    const uint64_t lp = static_cast<uint64_t>(j) * (kBN / 16) + pg;
                    uint64_t blk = __ldg(p.blocks + (lp < npages ? lp : 0));
                    if (blk >= p.num_blocks) {
                        raise_flag(p.status, KVFX_FLAG_BAD_INDEX);
                        blk = 0;
                    }
#pragma unroll
                    for (int b = 0; b < 2; ++b) {
                        tma_load_4d(kt + b * kKVHalf + pg * 2048, &kmap, b * 64, 0, static_cast<int>(kh),
                                    static_cast<int>(blk), &kv_full[st]);
                        tma_load_4d(vt + b * kKVHalf + pg * 2048, &vmap, b * 64, 0, static_cast<int>(kh),
                                    static_cast<int>(blk), &kv_full[st]);
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ----------------------------------------------------- MMA issuer ---
        if (lane == 0) {
            constexpr bool kBF = sizeof(T) == 2 && !std::is_same<T, __half>::value;
            const uint32_t id_qk = tc::idesc_f16(kBM, kBN, kBF, false);
            const uint32_t id_pv = tc::idesc_f16(kBM, kHD, kBF, true);
            bool ok = mbar_wait(&q_full, 0, p.status);
            auto issue_pv = [&](uint32_t jj) {
                const uint32_t vt = sbase + kOffV + (jj % kStages) * kKVTile;
#pragma unroll
                for (int part = 0; part < 2; ++part) {  // P_hi then P_lo
                    const uint32_t pa = sbase + (part == 0 ? kOffPHi : kOffPLo);
#pragma unroll
                    for (int t = 0; t < kBN / 16; ++t) {
                        tc::mma(tO, tc::desc_k_major(pa + t * 32), tc::desc_mn_major(vt + t * 2048, kKVHalf), id_pv,
                                (jj > 0 || part > 0 || t > 0) ? 1u : 0u);
                    }
                }
                tc::commit(&o_done);
                tc::commit(&kv_empty[jj % kStages]);
            };
            for (uint32_t j = 0; ok && j < ntiles; ++j) {
                const int st = static_cast<int>(j % kStages);
                if (!mbar_wait(&kv_full[st], (j / kStages) & 1u, p.status)) {
                    ok = false;
                    break;
                }
                if (j >= 2 && !mbar_wait(&s_empty[j & 1], ((j - 2) / 2) & 1u, p.status)) {
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                const uint32_t kt = sbase + kOffK + st * kKVTile;
#pragma unroll
                for (int part = 0; part < 2; ++part) {  // Q_hi then Q_lo
                    const uint32_t qa = sbase + (part == 0 ? kOffQHi : kOffQLo);
#pragma unroll
                    for (int kk = 0; kk < kHD / 16; ++kk) {
                        const uint32_t a = qa + (kk >> 2) * kQAtom + (kk & 3) * 32;
                        const uint32_t b = kt + (kk >> 2) * kKVHalf + (kk & 3) * 32;
                        tc::mma(tS[j & 1], tc::desc_k_major(a), tc::desc_k_major(b), id_qk,
                                (part > 0 || kk > 0) ? 1u : 0u);
                    }
                }
                tc::commit(&s_full[j & 1]);
                if (j >= 1) {
                    if (!mbar_wait(&p_full, (j - 1) & 1u, p.status)) {
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
                    issue_pv(j - 1);
                }
            }
            if (ok && ntiles > 0) {
                if (mbar_wait(&p_full, (ntiles - 1) & 1u, p.status)) {
                    tc::fence_after_sync();
                    issue_pv(ntiles - 1);
                } else {
                    ok = false;
                }
            }
            if (!ok) abort_flag = 1;
            // Every MMA this thread issued is complete before TMEM is released.
            tc::commit(&mma_done);
            (void)mbar_wait(&mma_done, 0, p.status);
        }
    } else {
        // -------------------------------------------------------- softmax ---
        const uint32_t quarter = static_cast<uint32_t>(warp & 3);  // TMEM lanes this warp may access
        const uint32_t r = quarter * 32 + lane;                     // query row within the tile
        const uint64_t qi = q0 + r;
        const bool row_live = qi < p.q_tokens;
        const uint64_t pos = p.kv_tokens - p.q_tokens + qi;         // last visible position
        const uint32_t lane_base = (quarter * 32) << 16;

        // Q row -> scaled hi/lo 16-bit halves in the swizzled K-major tiles.
        {
            const float* qrow = p.q + (qi * p.q_heads + qh) * kHD;
            unsigned char* qhi = smem + kOffQHi;
            unsigned char* qlo = smem + kOffQLo;
#pragma unroll 4
            for (uint32_t c = 0; c < kHD / 8; ++c) {
                float x[8];
                if (row_live) {
                    const float4 a = *reinterpret_cast<const float4*>(qrow + c * 8);
                    const float4 b = *reinterpret_cast<const float4*>(qrow + c * 8 + 4);
                    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
                    x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
                } else {
#pragma unroll
                    for (int e = 0; e < 8; ++e) x[e] = 0.f;
                }
                uint32_t hi[4], lo[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) split2<T>(x[2 * e] * p.qscale, x[2 * e + 1] * p.qscale, hi[e], lo[e]);
                const uint32_t off = (c >> 3) * kQAtom + swz_row(r, c & 7);
                *reinterpret_cast<uint4*>(qhi + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                *reinterpret_cast<uint4*>(qlo + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            }
            fence_proxy_async_smem();
            mbar_arrive(&q_full);
        }

        // tcgen05.ld/st are warp-collective: every wait result is made
        // warp-uniform so that no lane skips one the others execute.
        auto wait_all = [&](uint64_t* bar, uint32_t phase) {
            return __all_sync(0xffffffffu, mbar_wait(bar, phase, p.status)) != 0;
        };
        float m_run = -INFINITY, l_run = 0.f;
        bool ok = true;
        for (uint32_t j = 0; j < ntiles; ++j) {
            if (!wait_all(&s_full[j & 1], (j / 2) & 1u)) {
                ok = false;
                break;
            }
            tc::fence_after_sync();
            float s[kBN];
            tc::ld32(tS[j & 1] + lane_base, s);
            tc::ld32(tS[j & 1] + lane_base + 32, s + 32);
            tc::wait_ld();
            tc::fence_before_sync();
            mbar_arrive(&s_empty[j & 1]);

            const uint64_t t0 = static_cast<uint64_t>(j) * kBN;
            float mx = -INFINITY;
#pragma unroll
            for (int c = 0; c < kBN; ++c) {
                const uint64_t t = t0 + c;
                s[c] = (t <= pos && t < p.kv_tokens) ? s[c] : -INFINITY;
                mx = fmaxf(mx, s[c]);
            }
            // P's buffer (and O) are free once the previous tile's PV is done.
            if (j >= 1 && !wait_all(&o_done, (j - 1) & 1u)) {
                ok = false;
                break;
            }
            const bool need = mx > m_run + 8.f;  // m_run = -inf: always at tile 0
            const float m_new = need ? mx : m_run;
            const float alpha = exp2f(m_run - m_new);  // 1 if unchanged, 0 at the first tile
            if (j >= 1 && __any_sync(0xffffffffu, need)) {
                tc::fence_after_sync();
#pragma unroll 1
                for (int cb = 0; cb < kHD; cb += 32) {
                    float ov[32];
                    tc::ld32(tO + lane_base + cb, ov);
                    tc::wait_ld();
#pragma unroll
                    for (int e = 0; e < 32; ++e) ov[e] *= alpha;
                    tc::st32(tO + lane_base + cb, ov);
                }
                tc::wait_st();
            }
            l_run *= alpha;
            m_run = m_new;
            // P = exp2(S - m) as hi/lo halves in the swizzled K-major P tiles.
            unsigned char* phi = smem + kOffPHi;
            unsigned char* plo = smem + kOffPLo;
#pragma unroll
            for (int c = 0; c < kBN / 8; ++c) {
                uint32_t hi[4], lo[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float a = exp2f(s[c * 8 + 2 * e] - m_run);
                    const float b = exp2f(s[c * 8 + 2 * e + 1] - m_run);
                    l_run += a + b;
                    split2<T>(a, b, hi[e], lo[e]);
                }
                const uint32_t off = swz_row(r, c);
                *reinterpret_cast<uint4*>(phi + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                *reinterpret_cast<uint4*>(plo + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            }
            // Tokens past the sequence end in this tile: zero their V rows
            // (unwritten slots may hold NaN; 0 * NaN must not reach O).
            if (t0 + kBN > p.kv_tokens) {
                const uint32_t valid = static_cast<uint32_t>(p.kv_tokens - t0);
                const uint32_t rows = kBN - valid;
                unsigned char* vt = smem + kOffV + (j % kStages) * kKVTile;
                for (uint32_t x = r; x < rows * 2 * 8; x += 128) {
                    const uint32_t row = valid + x / 16, half = (x / 8) & 1, c = x & 7;
                    *reinterpret_cast<uint4*>(vt + half * kKVHalf + row * 128 + c * 16) = make_uint4(0, 0, 0, 0);
                }
            }
            fence_proxy_async_smem();
            tc::fence_before_sync();
            mbar_arrive(&p_full);
        }
        if (ok && ntiles > 0 && wait_all(&o_done, (ntiles - 1) & 1u)) {
            tc::fence_after_sync();
            const float inv = 1.f / l_run;
            float* orow = p.o + (qi * p.q_heads + qh) * kHD;
#pragma unroll 1
            for (int cb = 0; cb < kHD; cb += 32) {
                float ov[32];
                tc::ld32(tO + lane_base + cb, ov);
                tc::wait_ld();
                if (row_live) {
#pragma unroll
                    for (int e = 0; e < 32; e += 4) {
                        *reinterpret_cast<float4*>(orow + cb + e) =
                            make_float4(ov[e] * inv, ov[e + 1] * inv, ov[e + 2] * inv, ov[e + 3] * inv);
                    }
                }
            }
        } else if (!ok) {
            abort_flag = 1;
        }
    }

    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kTmemCols);
    }
}

bool prefill_eligible(const CacheView& c, const AttentionArgs& a) {
    return (c.dtype == KVFX_BF16 || c.dtype == KVFX_F16) && c.bs == 16 && c.hd == kHD && a.query_tokens >= 2 &&
           a.q_heads % c.heads == 0 && c.num_blocks < (1ull << 31) &&
           reinterpret_cast<uintptr_t>(a.q) % 16 == 0 && reinterpret_cast<uintptr_t>(a.o) % 16 == 0 &&
           ceil_div(a.query_tokens, kBM) < (1ull << 31) && a.q_heads <= 65535;
}

}  // namespace

bool prefill_tc_supported(const CacheView& c, const AttentionArgs& a) { return prefill_eligible(c, a); }

cudaError_t launch_prefill_tc(const CacheView& c, const AttentionArgs& a, unsigned* status, cudaStream_t s) {
    cudaError_t err = cudaSuccess;
    const CacheMaps* maps = cache_maps(c, &err);
    if (maps == nullptr) return err != cudaSuccess ? err : cudaErrorInvalidValue;
    static bool attr_done[64] = {false};
    const bool bf = c.dtype == KVFX_BF16;
    if (c.device < 0 || c.device >= 64 || !attr_done[c.device]) {
        err = cudaFuncSetAttribute(prefill_tc_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   kSmemAlloc);
        if (err != cudaSuccess) return err;
        err = cudaFuncSetAttribute(prefill_tc_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   kSmemAlloc);
        if (err != cudaSuccess) return err;
        if (c.device >= 0 && c.device < 64) attr_done[c.device] = true;
    }
    PrefillParams p;
    p.q = a.q;
    p.o = a.o;
    p.blocks = a.blocks;
    p.q_tokens = a.query_tokens;
    p.kv_tokens = a.kv_tokens;
    p.num_blocks = c.num_blocks;
    p.q_heads = a.q_heads;
    p.kv_heads = c.heads;
    p.group = a.q_heads / c.heads;
    p.n_qtiles = static_cast<uint32_t>(ceil_div(a.query_tokens, kBM));
    p.qscale = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(c.hd)));
    p.status = status;
    dim3 grid(p.n_qtiles, a.q_heads, 1);
    if (bf) {
        prefill_tc_kernel<__nv_bfloat16><<<grid, kThreads, kSmemAlloc, s>>>(p, maps->k, maps->v);
    } else {
        prefill_tc_kernel<__half><<<grid, kThreads, kSmemAlloc, s>>>(p, maps->k, maps->v);
    }
    return cudaGetLastError();
}

}  // namespace kvfx
