// Batch-decode PagedAttention (kernel 3).
//
// Work item = (split s, KV head h, request r): pages [s*P, (s+1)*P) of the
// request's block-table row, P = pages_per_split. The CTA's 4 warps take the
// item's pages round-robin; each warp streams its pages through a 2-stage
// shared-memory ring fed by TMA tensor loads (128-byte swizzle, no multicast),
// one 16-token K tile and V tile per page and KV head.
//
// GQA grouping: all G = Hq/Hkv query heads of KV head h are processed against
// each page, so every KV byte is read from HBM once. The math runs on
// mma.sync.m16n8k16 with FP32 accumulation; its 16 A-rows hold the G query
// heads twice: rows g carry the bf16/fp16 "hi" part of Q (and later of P),
// rows g+8 the "lo" residual, so hi+lo keeps ~16 mantissa bits of the FP32 Q
// and of the softmax weights and the result stays within FP32-class error of
// the reference's FP64 attention (KVFlux src/v2/paged_attention.cu:74-106).
// For G <= 8 the hi/lo rows cost no extra MMAs: the instruction has 16 rows.
//
// Softmax: online, base 2 (Q pre-scaled by log2(e)/sqrt(head_size)), with the
// running maximum only moved when a page's maximum exceeds it by more than 8
// (weights stay <= 2^8, exact in the hi/lo split), so the O accumulators are
// rescaled rarely. Rows of the last page beyond the sequence are masked to
// -inf in the scores and zeroed in the V tile (0 * garbage must not reach O).
//
// Split merge: a split writes (max, sum, unnormalised O) to the workspace and
// bumps a per-(request, head) counter; the CTA that completes the count resets
// the counter to zero, merges all splits with log-sum-exp weights and writes
// O. No CTA ever waits for another, and a workspace zero-filled once needs no
// clearing between launches (a CTA whose loads timed out still counts itself,
// with a split that contributes nothing, so every count completes).
//
// Append mode (one decode step fused with its paged KV write): each row's new
// token is the last position; the CTA whose split holds that page writes the
// new K/V row of its head into the cache, replaces the row in its shared-
// memory tiles, and takes the page from the token's slot, so the launch needs
// neither a separate write kernel nor a host update of the table.
#include <algorithm>
#include <atomic>
#include <cmath>

#include "common.cuh"
#include "launch.h"

namespace kvfx {


namespace {

constexpr int kWarps = 4;
constexpr int kStages = 2;
constexpr uint32_t kMaxSplits = 256;

struct DecodeParams {
    const float* q;
    float* o;
    const uint64_t* table;
    const uint64_t* lens;   // device lengths, or nullptr: every row has single_len
    uint64_t single_len;
    uint64_t max_blocks;
    uint64_t num_blocks;
    uint32_t kv_heads;
    uint32_t group;
    uint32_t pages_per_split;
    uint32_t max_splits;
    float qscale;
    float* partial;
    unsigned* counters;
    unsigned* status;
    // Append mode (all null for a plain decode): see DecodeArgs.
    const void* k_new;
    const void* v_new;
    const uint64_t* new_slots;
    uint64_t* table_out;
    char* k_base;
    char* v_base;
};

template <int HD>
struct Shape {
    static constexpr int kBoxes = HD / 64;               // 128-byte swizzle boxes per row
    static constexpr uint32_t kTile = 16u * HD * 2u;     // one 16-token tile, 16-bit elements
    static constexpr uint32_t kStage = 2u * kTile;       // K tile + V tile
    static constexpr int kKSteps = HD / 16;
    static constexpr int kNTiles = HD / 8;
    static constexpr uint32_t kSmem = kWarps * kStages * kStage + 1024;  // + alignment slack
    static constexpr uint32_t kPartial = 8u * (HD + 2);  // floats per split (8 head slots)
};

// Byte offset of the 16-byte chunk `c` (of HD/8) of token row `t` inside a
// tile stored as HD/64 boxes of [16 rows][128 B] with the TMA 128-byte swizzle
// (chunk index XOR row index mod 8).
__device__ __forceinline__ uint32_t swz(int t, int c) {
    return static_cast<uint32_t>((c >> 3) * 2048 + t * 128 + (((c & 7) ^ (t & 7)) << 4));
}

template <int HD, typename T>
__global__ void __launch_bounds__(kWarps * 32, 3)
decode_mma_kernel(const __grid_constant__ DecodeParams p, const __grid_constant__ CUtensorMap kmap,
                  const __grid_constant__ CUtensorMap vmap) {
    using S = Shape<HD>;
    extern __shared__ unsigned char smem_raw[];
    __shared__ uint64_t bars[kWarps][kStages];
    __shared__ float s_m[kWarps][8], s_l[kWarps][8];
    __shared__ float s_scale[kWarps][8], s_inv[8];
    __shared__ int s_flag;

    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t split = blockIdx.x, kh = blockIdx.y;
    const uint64_t r = blockIdx.z;

    // Launched as a programmatic dependent: the stream's next kernel may be
    // scheduled as soon as every CTA of this one has started (so its CTAs
    // take the SMs this launch's last wave leaves), and this one reads
    // nothing before the kernel ahead of it has completed.
    pdl_allow_next();
    pdl_wait();
    const uint64_t len = p.lens != nullptr ? p.lens[r] : p.single_len;
    const uint64_t npages = ceil_div(len, 16);
    const uint32_t nsplits = static_cast<uint32_t>(ceil_div(npages, p.pages_per_split));
    if (len == 0 || split >= nsplits) return;
    if (nsplits > p.max_splits || npages > p.max_blocks) {  // length beyond the host's bounds: refuse
        if (tid == 0) raise_flag(p.status, KVFX_FLAG_BAD_INDEX);
        return;
    }
    const uint64_t pbeg = static_cast<uint64_t>(split) * p.pages_per_split;
    const uint64_t pend = umin64(npages, pbeg + p.pages_per_split);
    const uint64_t* row = p.table + r * p.max_blocks;
    const uint32_t n_my =
        pend > pbeg + warp ? static_cast<uint32_t>(ceil_div(pend - pbeg - warp, kWarps)) : 0u;
    unsigned char* wsm = smem + static_cast<size_t>(warp) * kStages * S::kStage;

    // Append mode: the CTA holding the row's last page writes this head's
    // new K/V row into the cache and into that page's tiles once they land
    // (so the TMA load may see the old or the new row: either is replaced),
    // and loads the page the slot names in place of the table entry. No
    // other CTA reads that table entry in this launch; the head-0 CTA stores
    // the page there for later launches.
    const bool append = p.k_new != nullptr;
    const uint64_t last = npages - 1;
    uint64_t new_blk = ~0ull;
    uint32_t new_row = 0;
    if (append && split == nsplits - 1) {
        const uint64_t slot = p.new_slots[r];
        if ((slot >> 4) < p.num_blocks && (slot & 15u) == ((len - 1) & 15u)) {
            new_blk = slot >> 4;
            new_row = static_cast<uint32_t>(slot & 15u);
        } else if (tid == 0) {
            raise_flag(p.status, KVFX_FLAG_BAD_INDEX);
        }
    }
    const bool owns_new = new_blk != ~0ull && static_cast<uint32_t>((last - pbeg) % kWarps) == warp;
    constexpr int kRowChunks = HD / 8;  // 16-byte chunks of one (token, head) row
    uint4 new_chunk = make_uint4(0, 0, 0, 0);
    if (owns_new) {
        if (lane < 2 * kRowChunks) {
            const bool isv = lane >= kRowChunks;
            const int c = isv ? lane - kRowChunks : lane;
            const uint64_t row_off = ((r * p.kv_heads + kh) * HD) * 2 + static_cast<uint64_t>(c) * 16;
            new_chunk = __ldg(reinterpret_cast<const uint4*>(static_cast<const char*>(isv ? p.v_new : p.k_new) +
                                                             row_off));
            const uint64_t dst = (((new_blk * p.kv_heads + kh) * 16 + new_row) * HD) * 2 + static_cast<uint64_t>(c) * 16;
            *reinterpret_cast<uint4*>((isv ? p.v_base : p.k_base) + dst) = new_chunk;
        }
        if (kh == 0 && lane == 0) p.table_out[r * p.max_blocks + last] = new_blk;
    }

    if (lane == 0) {
        for (int st = 0; st < kStages; ++st) mbar_init(&bars[warp][st], 1);
        fence_mbarrier_init();
        prefetch_tensormap(&kmap);
        prefetch_tensormap(&vmap);
    }
    __syncwarp();

    // This warp's page ids, read once up front: lane l holds those of its
    // pages l and l + 32 (splits of up to 64 pages per warp; longer ones read
    // each id when its page is issued), so a ring slot's refill does not wait
    // for a table read.
    const bool ids_cached = n_my <= 64;
    uint64_t id_lo = 0, id_hi = 0;
    if (ids_cached) {
        const uint64_t j0 = pbeg + warp + static_cast<uint64_t>(kWarps) * lane;
        const uint64_t j1 = j0 + static_cast<uint64_t>(kWarps) * 32;
        if (lane < n_my) id_lo = append ? __ldcg(row + j0) : __ldg(row + j0);
        if (lane + 32 < n_my) id_hi = append ? __ldcg(row + j1) : __ldg(row + j1);
    }
    auto issue = [&](uint32_t i) {  // whole warp; lane 0 issues the copies of page i of this warp
        if (i >= n_my) return;
        const uint64_t j = pbeg + warp + static_cast<uint64_t>(kWarps) * i;
        uint64_t blk;
        if (ids_cached) {
            blk = __shfl_sync(0xffffffffu, i < 32 ? id_lo : id_hi, i & 31);
        } else if (lane == 0) {
            blk = append ? __ldcg(row + j) : __ldg(row + j);
        } else {
            blk = 0;
        }
        if (append && j == last && new_blk != ~0ull) blk = new_blk;
        if (lane != 0) return;
        if (blk >= p.num_blocks) {
            raise_flag(p.status, KVFX_FLAG_BAD_INDEX);
            blk = 0;
        }
        const int st = static_cast<int>(i % kStages);
        unsigned char* kt = wsm + st * S::kStage;
        mbar_arrive_expect_tx(&bars[warp][st], S::kStage);
#pragma unroll
        for (int b = 0; b < S::kBoxes; ++b) {
            tma_load_4d(kt + b * 2048, &kmap, b * 64, 0, static_cast<int>(kh), static_cast<int>(blk),
                        &bars[warp][st]);
            tma_load_4d(kt + S::kTile + b * 2048, &vmap, b * 64, 0, static_cast<int>(kh),
                        static_cast<int>(blk), &bars[warp][st]);
        }
    };
#pragma unroll
    for (int i = 0; i < kStages; ++i) issue(i);

    // Q fragments (A operand): rows g = hi(Q[g]), rows g+8 = lo(Q[g]).
    const int g = lane >> 2, tig = lane & 3;
    const bool live = static_cast<uint32_t>(g) < p.group;
    uint32_t qa[S::kKSteps][4];
    {
        const uint64_t qh = static_cast<uint64_t>(kh) * p.group + (live ? g : 0);
        const float* qrow = p.q + (r * p.kv_heads * p.group + qh) * HD;
#pragma unroll
        for (int kk = 0; kk < S::kKSteps; ++kk) {
            const int c0 = 16 * kk + 2 * tig;
            const float x0 = live ? qrow[c0] * p.qscale : 0.f;
            const float x1 = live ? qrow[c0 + 1] * p.qscale : 0.f;
            const float x8 = live ? qrow[c0 + 8] * p.qscale : 0.f;
            const float x9 = live ? qrow[c0 + 9] * p.qscale : 0.f;
            split2<T>(x0, x1, qa[kk][0], qa[kk][1]);
            split2<T>(x8, x9, qa[kk][2], qa[kk][3]);
        }
    }

    float m_run = -INFINITY, l_run = 0.f;
    float oacc[S::kNTiles][4];
#pragma unroll
    for (int n = 0; n < S::kNTiles; ++n) oacc[n][0] = oacc[n][1] = oacc[n][2] = oacc[n][3] = 0.f;

    bool ok = true;
    for (uint32_t i = 0; i < n_my; ++i) {
        const int st = static_cast<int>(i % kStages);
        if (!mbar_wait(&bars[warp][st], (i / kStages) & 1u, p.status)) {
            ok = false;
            break;
        }
        unsigned char* ktp = wsm + st * S::kStage;
        const uint32_t kt = smem_addr(ktp), vt = kt + S::kTile;
        const uint64_t tok0 = (pbeg + warp + static_cast<uint64_t>(kWarps) * i) * 16;
        const int valid = static_cast<int>(umin64(16, len - tok0));
        if (owns_new && tok0 + 16 >= len) {  // this warp's last page holds the new token
            if (lane < 2 * kRowChunks) {
                const bool isv = lane >= kRowChunks;
                const int c = isv ? lane - kRowChunks : lane;
                *reinterpret_cast<uint4*>(ktp + (isv ? S::kTile : 0u) + swz(static_cast<int>(new_row), c)) =
                    new_chunk;
            }
            __syncwarp();
        }
        if (valid < 16) {
            // Zero V rows past the sequence end (they may hold anything).
            uint4* vz = reinterpret_cast<uint4*>(ktp + S::kTile);
            const int chunks = (16 - valid) * 8;  // 16-byte chunks per box
#pragma unroll
            for (int b = 0; b < S::kBoxes; ++b) {
                for (int x = lane; x < chunks; x += 32) {
                    vz[(b * 2048 + valid * 128) / 16 + x] = make_uint4(0, 0, 0, 0);
                }
            }
            __syncwarp();
        }

        // S = Q K^T for 16 tokens (two n-tiles of 8).
        float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        {
            const int mi = lane >> 3, jr = lane & 7;
            const int t = (mi >> 1) * 8 + jr;
#pragma unroll
            for (int kk = 0; kk < S::kKSteps; ++kk) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4(kt + swz(t, 2 * kk + (mi & 1)), b0, b1, b2, b3);
                MmaKind<T>::mma(sc[0], qa[kk], b0, b1);
                MmaKind<T>::mma(sc[1], qa[kk], b2, b3);
            }
        }
        float s[2][2];
        float mx = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int t = 8 * nt + 2 * tig + e;
                const float v = sc[nt][e] + sc[nt][2 + e];
                s[nt][e] = t < valid ? v : -INFINITY;
                mx = fmaxf(mx, s[nt][e]);
            }
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const bool need = mx > m_run + 8.f;
        if (__any_sync(0xffffffffu, need)) {
            const float m_new = need ? mx : m_run;
            const float alpha = exp2f(m_run - m_new);
            l_run *= alpha;
#pragma unroll
            for (int n = 0; n < S::kNTiles; ++n) {
                oacc[n][0] *= alpha;
                oacc[n][1] *= alpha;
                oacc[n][2] *= alpha;
                oacc[n][3] *= alpha;
            }
            m_run = m_new;
        }
        float pw[2][2];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
            pw[nt][0] = exp2f(s[nt][0] - m_run);
            pw[nt][1] = exp2f(s[nt][1] - m_run);
            l_run += pw[nt][0] + pw[nt][1];
        }
        uint32_t pa[4];
        split2<T>(pw[0][0], pw[0][1], pa[0], pa[1]);
        split2<T>(pw[1][0], pw[1][1], pa[2], pa[3]);

        // O += P V over 16 tokens, HD/8 n-tiles of 8 dimensions.
        {
            const int mi = lane >> 3, jr = lane & 7;
            const int t = (mi & 1) * 8 + jr;
#pragma unroll
            for (int n2 = 0; n2 < S::kNTiles / 2; ++n2) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(vt + swz(t, 2 * n2 + (mi >> 1)), b0, b1, b2, b3);
                MmaKind<T>::mma(oacc[2 * n2], pa, b0, b1);
                MmaKind<T>::mma(oacc[2 * n2 + 1], pa, b2, b3);
            }
        }
        __syncwarp();
        issue(i + kStages);
    }

    // ---- combine the 4 warps of this CTA (stage memory is free again) ----
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
    if (tid == 0) s_flag = 0;
    __syncthreads();
    if (!ok) s_flag = 1;
    __syncthreads();
    // A load never arrived (status already flagged): no O from this CTA; a
    // split still counts itself with an empty partial (below).
    const bool failed = s_flag != 0;
    if (failed && nsplits == 1) return;

    float* mo = reinterpret_cast<float*>(smem);  // [kWarps][8][HD]
    if (!failed) {
        if (live) {
            float* dst = mo + (warp * 8 + g) * HD;
#pragma unroll
            for (int n = 0; n < S::kNTiles; ++n) {
                *reinterpret_cast<float2*>(dst + 8 * n + 2 * tig) =
                    make_float2(oacc[n][0] + oacc[n][2], oacc[n][1] + oacc[n][3]);
            }
            if (tig == 0) {
                s_m[warp][g] = m_run;
                s_l[warp][g] = l_run;
            }
        } else if (tig == 0) {
            s_m[warp][g] = -INFINITY;
            s_l[warp][g] = 0.f;
        }
    }
    __syncthreads();
    const uint32_t G = p.group;
    if (!failed && tid < static_cast<int>(G)) {
        float M = -INFINITY;
        for (int w = 0; w < kWarps; ++w) M = fmaxf(M, s_m[w][tid]);
        float L = 0.f;
        for (int w = 0; w < kWarps; ++w) {
            const float f = s_m[w][tid] == -INFINITY ? 0.f : exp2f(s_m[w][tid] - M);
            s_scale[w][tid] = f;
            L += s_l[w][tid] * f;
        }
        s_m[0][tid] = M;  // reuse: CTA max and sum
        s_l[0][tid] = L;
        s_inv[tid] = 1.f / L;
    }
    __syncthreads();

    const uint64_t pair = r * p.kv_heads + kh;
    if (nsplits == 1) {
        for (uint32_t idx = tid; idx < G * HD; idx += kWarps * 32) {
            const uint32_t gg = idx / HD, d = idx - gg * HD;
            float acc = 0.f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) acc += mo[(w * 8 + gg) * HD + d] * s_scale[w][gg];
            p.o[(r * p.kv_heads * G + static_cast<uint64_t>(kh) * G + gg) * HD + d] = acc * s_inv[gg];
        }
        return;
    }

    float* part = p.partial + (pair * p.max_splits + split) * static_cast<uint64_t>(S::kPartial);
    for (uint32_t idx = tid; idx < G * HD; idx += kWarps * 32) {
        const uint32_t gg = idx / HD, d = idx - gg * HD;
        float acc = 0.f;
        if (!failed) {
#pragma unroll
            for (int w = 0; w < kWarps; ++w) acc += mo[(w * 8 + gg) * HD + d] * s_scale[w][gg];
        }
        part[gg * (HD + 2) + d] = acc;
    }
    if (tid < static_cast<int>(G)) {
        part[tid * (HD + 2) + HD] = failed ? -INFINITY : s_m[0][tid];
        part[tid * (HD + 2) + HD + 1] = failed ? 0.f : s_l[0][tid];
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        // 16-bit counters, two per word; nsplits <= 256 never carries.
        unsigned* word = p.counters + (pair >> 1);
        const unsigned shift = static_cast<unsigned>(pair & 1u) * 16u;
        const unsigned prev = (atomicAdd(word, 1u << shift) >> shift) & 0xffffu;
        const bool last = prev == nsplits - 1;
        if (last) atomicSub(word, nsplits << shift);  // zero again for the next launch
        s_flag = last ? 2 : 0;
    }
    __syncthreads();
    if (s_flag != 2) return;
    __threadfence();

    // Last split to finish: merge every split of this (request, head).
    float* wsplit = reinterpret_cast<float*>(smem);  // [8][kMaxSplits] weights
    const float* base = p.partial + pair * p.max_splits * static_cast<uint64_t>(S::kPartial);
    if (tid < static_cast<int>(G)) {
        float M = -INFINITY;
        for (uint32_t sp = 0; sp < nsplits; ++sp) {
            M = fmaxf(M, __ldcg(base + sp * S::kPartial + tid * (HD + 2) + HD));
        }
        float L = 0.f;
        for (uint32_t sp = 0; sp < nsplits; ++sp) {
            const float* ps = base + sp * S::kPartial + tid * (HD + 2);
            const float f = exp2f(__ldcg(ps + HD) - M);
            wsplit[tid * kMaxSplits + sp] = f;
            L += __ldcg(ps + HD + 1) * f;
        }
        s_inv[tid] = 1.f / L;
    }
    __syncthreads();
    for (uint32_t idx = tid; idx < G * HD; idx += kWarps * 32) {
        const uint32_t gg = idx / HD, d = idx - gg * HD;
        float acc = 0.f;
        for (uint32_t sp = 0; sp < nsplits; ++sp) {
            acc += __ldcg(base + sp * S::kPartial + gg * (HD + 2) + d) * wsplit[gg * kMaxSplits + sp];
        }
        p.o[(r * p.kv_heads * G + static_cast<uint64_t>(kh) * G + gg) * HD + d] = acc * s_inv[gg];
    }
}

// Append step for the shapes the fast kernel does not cover, ahead of the
// generic attention launch: one CTA per row validates the new token's slot
// against its position, stores the slot's page into the table and copies the
// row's K/V for every head (element-wise).
template <typename E>
__global__ void append_rows_kernel(char* k, char* v, const void* k_new, const void* v_new,
                                   const uint64_t* new_slots, uint64_t* table, const uint64_t* lens,
                                   uint64_t max_blocks, uint64_t num_blocks, uint32_t heads, uint32_t bs,
                                   uint32_t hd, unsigned* status) {
    const uint64_t r = blockIdx.x;
    const uint64_t len = lens[r];
    const uint64_t slot = new_slots[r];
    const uint64_t blk = slot / bs, off = slot % bs;
    if (len == 0 || (len - 1) / bs >= max_blocks || blk >= num_blocks || off != (len - 1) % bs) {
        if (threadIdx.x == 0) raise_flag(status, KVFX_FLAG_BAD_INDEX);
        return;
    }
    if (threadIdx.x == 0) table[r * max_blocks + (len - 1) / bs] = blk;
    const uint64_t n = static_cast<uint64_t>(heads) * hd;
    const E* ks = static_cast<const E*>(k_new) + r * n;
    const E* vs = static_cast<const E*>(v_new) + r * n;
    for (uint64_t x = threadIdx.x; x < n; x += blockDim.x) {
        const uint64_t h = x / hd, d = x - h * hd;
        const uint64_t dst = ((blk * heads + h) * bs + off) * hd + d;
        reinterpret_cast<E*>(k)[dst] = ks[x];
        reinterpret_cast<E*>(v)[dst] = vs[x];
    }
}

bool fast_path(const CacheView& c, uint32_t group) {
    return (c.dtype == KVFX_BF16 || c.dtype == KVFX_F16) && c.bs == 16 &&
           (c.hd == 64 || c.hd == 128) && group >= 1 && group <= 8 &&
           c.num_blocks < (1ull << 31) && c.heads < (1u << 31);
}

template <int HD, typename T>
cudaError_t launch_fast(const CacheView& c, const DecodeArgs& a, const CacheMaps* maps, uint32_t pps,
                        uint32_t max_splits, unsigned* status, cudaStream_t s) {
    using Sh = Shape<HD>;
    static std::atomic<int> attr_done[64];  // zero-initialised (static storage)
    if (c.device < 0 || c.device >= 64 || !attr_done[c.device].load(std::memory_order_acquire)) {
        // Idempotent: threads that race here all set the same attribute.
        cudaError_t e = cudaFuncSetAttribute(decode_mma_kernel<HD, T>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, Sh::kSmem);
        if (e != cudaSuccess) return e;
        if (c.device >= 0 && c.device < 64) attr_done[c.device].store(1, std::memory_order_release);
    }
    DecodeParams p;
    p.q = a.q;
    p.o = a.o;
    p.table = a.table;
    p.lens = a.lens;
    p.single_len = a.max_len;
    p.max_blocks = a.max_blocks;
    p.num_blocks = c.num_blocks;
    p.kv_heads = c.heads;
    p.group = a.q_heads / c.heads;
    p.pages_per_split = pps;
    p.max_splits = max_splits;
    p.qscale = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(c.hd)));
    p.counters = static_cast<unsigned*>(a.workspace);
    p.partial = reinterpret_cast<float*>(static_cast<char*>(a.workspace) + decode_counter_bytes(c.heads));
    p.status = status;
    p.k_new = a.k_new;
    p.v_new = a.v_new;
    p.new_slots = a.new_slots;
    p.table_out = a.table_out;
    p.k_base = c.k;
    p.v_base = c.v;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(max_splits, c.heads, static_cast<uint32_t>(a.batch));
    cfg.blockDim = dim3(kWarps * 32);
    cfg.dynamicSmemBytes = Sh::kSmem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, decode_mma_kernel<HD, T>, p, maps->k, maps->v);
}

uint32_t clamp_pps(const CacheView& c, uint64_t max_len, uint32_t pps) {
    const uint64_t max_pages = ceil_div(std::max<uint64_t>(max_len, 1), c.bs);
    uint64_t lo = std::max<uint64_t>(kWarps, ceil_div(max_pages, kMaxSplits));
    uint64_t v = std::max<uint64_t>(pps, lo);
    v = ceil_div(v, kWarps) * kWarps;
    return static_cast<uint32_t>(std::min<uint64_t>(v, 1u << 30));
}

}  // namespace

uint32_t decode_pages_per_split(const CacheView& c, uint64_t batch, uint32_t q_heads, uint64_t max_len,
                                uint64_t total_tokens) {
    (void)q_heads;
    // Splits as long as possible while about three waves of CTAs (3 per SM)
    // remain: each split pays a fixed cost (ring start, Q staging, partials,
    // merge) that outweighs the shorter tail of finer splits. Measured on
    // B200 (ms per launch): config 5 at 1 GPU 2.643 / 2.616 with 128 / 256
    // pages; its 8-way shard 0.378 / 0.369 with 80 / 192; config 3
    // 0.1946 / 0.186 with 40 / 96.
    const uint64_t tokens = total_tokens != 0 ? total_tokens : batch * max_len;
    const uint64_t page_heads = ceil_div(tokens, c.bs) * c.heads;
    const uint64_t target = static_cast<uint64_t>(device_sm_count(c.device)) * 3 * 3;
    uint64_t pps = page_heads / std::max<uint64_t>(target, 1);
    pps = std::min<uint64_t>(std::max<uint64_t>(pps, 8), 256);
    return clamp_pps(c, max_len, static_cast<uint32_t>(pps));
}

uint64_t decode_workspace_bytes(const CacheView& c, uint64_t batch, uint32_t q_heads, uint64_t max_len,
                                uint32_t pages_per_split) {
    const uint32_t group = c.heads ? q_heads / c.heads : 0;
    if (!fast_path(c, group)) return 0;
    if (pages_per_split == 0) pages_per_split = decode_pages_per_split(c, batch, q_heads, max_len, 0);
    const uint32_t pps = clamp_pps(c, max_len, pages_per_split);
    const uint64_t max_splits = ceil_div(ceil_div(std::max<uint64_t>(max_len, 1), c.bs), pps);
    const uint64_t per = 8ull * (c.hd + 2);
    const uint64_t pbytes = ((batch * c.heads * max_splits * per * 4) + 255) & ~uint64_t(255);
    return decode_counter_bytes(c.heads) + pbytes;
}

cudaError_t launch_decode(const CacheView& c, const DecodeArgs& a, unsigned* status, cudaStream_t s) {
    const uint32_t group = a.q_heads / c.heads;
    const bool append = a.k_new != nullptr;
    const bool aligned = !append || ((reinterpret_cast<uintptr_t>(a.k_new) | reinterpret_cast<uintptr_t>(a.v_new)) & 15u) == 0;
    if (!fast_path(c, group) || !aligned) {
        if (append) {
            if (c.elem == 4) {
                append_rows_kernel<uint32_t><<<static_cast<uint32_t>(a.batch), 128, 0, s>>>(
                    c.k, c.v, a.k_new, a.v_new, a.new_slots, a.table_out, a.lens, a.max_blocks, c.num_blocks,
                    c.heads, c.bs, c.hd, status);
            } else {
                append_rows_kernel<uint16_t><<<static_cast<uint32_t>(a.batch), 128, 0, s>>>(
                    c.k, c.v, a.k_new, a.v_new, a.new_slots, a.table_out, a.lens, a.max_blocks, c.num_blocks,
                    c.heads, c.bs, c.hd, status);
            }
            const cudaError_t e = cudaGetLastError();
            if (e != cudaSuccess) return e;
        }
        GenericAttnArgs g{a.q, a.o, a.table, a.max_blocks, a.lens, a.batch, 0, a.q_heads};
        return launch_attention_generic(c, g, status, s);
    }
    cudaError_t err = cudaSuccess;
    const CacheMaps* maps = cache_maps(c, &err);
    if (maps == nullptr) return err != cudaSuccess ? err : cudaErrorInvalidValue;
    uint32_t pps = a.pages_per_split != 0 ? a.pages_per_split
                                          : decode_pages_per_split(c, a.batch, a.q_heads, a.max_len, 0);
    pps = clamp_pps(c, a.max_len, pps);
    const uint32_t max_splits =
        static_cast<uint32_t>(ceil_div(ceil_div(std::max<uint64_t>(a.max_len, 1), c.bs), pps));
    if (c.hd == 128) {
        return c.dtype == KVFX_BF16
                   ? launch_fast<128, __nv_bfloat16>(c, a, maps, pps, max_splits, status, s)
                   : launch_fast<128, __half>(c, a, maps, pps, max_splits, status, s);
    }
    return c.dtype == KVFX_BF16 ? launch_fast<64, __nv_bfloat16>(c, a, maps, pps, max_splits, status, s)
                                : launch_fast<64, __half>(c, a, maps, pps, max_splits, status, s);
}

cudaError_t launch_decode_with_maps(const CacheView& c, const DecodeArgs& a, const CacheMaps& maps,
                                    unsigned* status, cudaStream_t s) {
    const uint32_t group = a.q_heads / c.heads;
    if (!fast_path(c, group)) return cudaErrorInvalidValue;
    const uint32_t pps = clamp_pps(c, a.max_len, a.pages_per_split);
    const uint32_t max_splits =
        static_cast<uint32_t>(ceil_div(ceil_div(std::max<uint64_t>(a.max_len, 1), c.bs), pps));
    if (c.hd == 128) {
        return c.dtype == KVFX_BF16
                   ? launch_fast<128, __nv_bfloat16>(c, a, &maps, pps, max_splits, status, s)
                   : launch_fast<128, __half>(c, a, &maps, pps, max_splits, status, s);
    }
    return c.dtype == KVFX_BF16 ? launch_fast<64, __nv_bfloat16>(c, a, &maps, pps, max_splits, status, s)
                                : launch_fast<64, __half>(c, a, &maps, pps, max_splits, status, s);
}

}  // namespace kvfx
