// Causal prefill PagedAttention on the 5th-generation tensor cores (kernel 4).
//
// Persistent: one CTA per SM walks a list of work units, one unit = a query
// tile of 128 rows of one Q head against the KV tiles of 128 tokens (8 pages)
// that its rows can see. Units are ordered heaviest first (last query tiles
// first) and dealt to CTAs in snake order (round r: CTA c takes unit
// r*G + c, or r*G + G-1-c on odd rounds), which evens out the causal
// triangle's unequal work. Tiles of consecutive units form one stream per
// CTA, so loads, MMAs and softmax run across unit boundaries without a drain.
// Warp roles (12 warps):
//   warp 0      K producer, warp 2 V producer: per KV tile 16 tensor loads
//               (8 pages x 2 64-dim halves, 128-byte swizzle, no multicast)
//               into a 4-slot K ring and a 2-slot V ring.
//   warp 1      owns TMEM (512 columns) and issues every tcgen05.mma from one
//               thread: S(g) = Q K_g^T into S[g%2] with Q read from TMEM, then
//               O += P(g) V_g with P read from TMEM; QK runs two tiles ahead
//               of PV.
//   warp 3      idle.
//   warps 4-7   softmax, one query row per thread (TMEM lane = row): scores
//               from TMEM, causal mask, online softmax in base 2, P = exp2(S-m)
//               written back over its own S columns as packed 16-bit hi/lo
//               pairs; at a unit's last tile, the row sums l go to shared
//               memory and the softmax moves straight on to the next unit.
//   warps 8-11  Q staging and epilogue: the next unit's Q rows are loaded
//               into registers while the current unit runs, and written as
//               hi/lo 16-bit halves into the Q columns of TMEM once its last
//               QK has completed; then the unit's O is read from TMEM (O is
//               released to the next unit's first PV as soon as it is in
//               registers) and O / l is written to global memory, off the
//               softmax's critical path.
// TMEM columns: S/P buffers 0 and 128; O 256; Q 384 (hi 384..447, lo
// 448..511). S[g%2] holds P(g) until PV(g) has read it; QK(g+2), which
// overwrites it, is issued after PV(g) by the same thread, and tcgen05.mma
// operations issued by one thread execute in issue order, so PV(g) has read
// P(g) before QK(g+2) writes there (no wait in between; the tensor pipe
// stays busy). Q in TMEM halves the shared-memory operand traffic of QK
// (only K is read from shared memory), the resource that bounded the
// tile rate when both operands came from there.
// Precision: Q (FP32 in the API) and P are each fed as two 16-bit operands,
// hi = round(x) and lo = round(x - hi), accumulated into the same TMEM tile
// (S = Q_hi K + Q_lo K, O += P_hi V + P_lo V): ~16 mantissa bits and FP32-class
// error against the FP64 reference; rounding Q or P to 16 bits alone exceeds
// 2e-3 at 4096 tokens. O is rescaled in TMEM only when a tile's row maximum
// exceeds the running one by more than 8 (base-2 units). Tokens past the
// sequence end in the last tile are masked in S and zeroed in the V tile.
//
// Semantics: KVFlux src/v2/paged_attention.cu:109-128 (query i sees
// positions <= kv_tokens - query_tokens + i; KV head = q_head / group).
#include <algorithm>
#include <atomic>
#include <cmath>
#include <type_traits>

#include "common.cuh"
#include "launch.h"
#include "tcgen05.cuh"

namespace kvfx {
namespace {

constexpr int kBM = 128;         // query rows per unit
constexpr int kBN = 128;         // KV tokens per tile (8 pages of 16)
constexpr int kHD = 128;         // head size handled here
constexpr uint32_t kMaxPrefillSeqs = KVFX_MAX_PREFILL_SEQS;  // sequences per launch
constexpr int kKStages = 4;      // K ring depth
constexpr int kVStages = 2;      // V ring depth
constexpr int kSBufs = 2;        // S/P buffers in TMEM
constexpr int kThreads = 384;    // 12 warps
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemO = kSBufs * kBN;          // O accumulator column
constexpr uint32_t kTmemQ = kTmemO + kHD;          // Q: hi pairs, then lo pairs (64 columns each)
static_assert(kTmemQ + kHD == kTmemCols, "TMEM budget");
// The V producer's waits on pv_done rely on a ring of no more slots than
// there are S buffers (see produce()); the K ring has its own free barriers.
static_assert(kVStages <= kSBufs, "V ring deeper than the S buffers");

// Shared-memory layout (byte offsets from a 1024-aligned base).
constexpr uint32_t kKVHalf = kBN * 128;            // [128 tokens][64 dims], 16 KiB
constexpr uint32_t kKVTile = 2 * kKVHalf;          // 32 KiB
constexpr uint32_t kOffK = 0;
constexpr uint32_t kOffV = kOffK + kKStages * kKVTile;
constexpr uint32_t kSmemBytes = kOffV + kVStages * kKVTile;   // 192 KiB
constexpr uint32_t kSmemAlloc = kSmemBytes + 1024;

// One sequence of a launch: its Q and O ([q_tokens][q_heads][128] FP32), its
// page ids and its lengths.
struct PrefillSeq {
    const float* q;
    float* o;
    const uint64_t* blocks;
    uint64_t q_tokens, kv_tokens;
};

struct PrefillParams {
    PrefillSeq seq[kMaxPrefillSeqs];
    uint64_t num_blocks;
    uint32_t n_units;  // max query tiles x sequences x Q heads (shorter sequences leave gaps), < 2^31
    uint32_t num_seqs, q_heads, kv_heads, group;
    FastDiv div_round, div_qheads, div_group;  // by num_seqs x q_heads, q_heads, group
    float qscale;
    unsigned* status;
};

struct Unit {
    uint64_t q0;
    uint32_t qh, kh, ntiles, s;
};

// The unit this CTA takes in dealing round `round` (false when it has none
// left). Unit index = (unit round, sequence, Q head); unit round 0 holds
// every sequence's last query tile, so the heaviest units come first across
// sequences; an index past a shorter sequence's first tile is a gap, and the
// CTA moves on to its next round (every role calls this with its own round
// counter and skips the same gaps).
// Inlined in every role, so kept small: unit indices stay below 2^31 (the
// host checks) and the three divisions are multiply-highs by constants the
// host prepares.
__device__ __forceinline__ bool unit_at(const PrefillParams& p, uint32_t& round, Unit& u) {
    const uint32_t G = gridDim.x;
    for (;; ++round) {
        const uint64_t base = static_cast<uint64_t>(round) * G;
        if (base >= p.n_units) return false;
        const uint32_t idx = static_cast<uint32_t>(base) + ((round & 1u) ? (G - 1 - blockIdx.x) : blockIdx.x);
        if (idx >= p.n_units) return false;  // partial last round
        const uint32_t ur = fast_div(idx, p.div_round);
        const uint32_t rem = idx - ur * (p.num_seqs * p.q_heads);
        u.s = fast_div(rem, p.div_qheads);
        u.qh = rem - u.s * p.q_heads;
        const PrefillSeq& sq = p.seq[u.s];
        const uint64_t nq = ceil_div(sq.q_tokens, kBM);
        if (ur >= nq) continue;
        u.kh = fast_div(u.qh, p.div_group);
        u.q0 = (nq - 1 - ur) * kBM;
        const uint64_t q_last = umin64(u.q0 + kBM, sq.q_tokens) - 1;
        u.ntiles = static_cast<uint32_t>((sq.kv_tokens - sq.q_tokens + q_last) / kBN + 1);
        return true;
    }
}

// Position in this CTA's stream of KV tiles: unit ordinal k, tile j of the
// unit, and the running tile ordinal g that indexes rings and barriers.
struct TileCursor {
    Unit u;
    uint32_t round, k, j, g;
    bool valid;
    __device__ __forceinline__ void init(const PrefillParams& p) {
        round = k = j = g = 0;
        valid = unit_at(p, round, u);
    }
    __device__ __forceinline__ void next(const PrefillParams& p) {
        ++g;
        if (++j < u.ntiles) return;
        j = 0;
        ++k;
        ++round;
        valid = unit_at(p, round, u);
    }
    __device__ __forceinline__ bool last() const { return j + 1 == u.ntiles; }
};

// The two 16-bit values of a packed pair, widened to float (low half first).
template <typename T>
__device__ __forceinline__ uint64_t widen2(uint32_t h);
template <>
__device__ __forceinline__ uint64_t widen2<__nv_bfloat16>(uint32_t h) {
    return f2_pack(__uint_as_float(h << 16), __uint_as_float(h & 0xFFFF0000u));
}
template <>
__device__ __forceinline__ uint64_t widen2<__half>(uint32_t h) {
    const __half2 x = *reinterpret_cast<const __half2*>(&h);
    return f2_pack(__low2float(x), __high2float(x));
}

// Page id of page `lane` of KV tile j of sequence s in lanes 0..7 (one load
// per lane, all in one memory round trip); 0 in the other lanes.
__device__ __forceinline__ uint64_t tile_page_id(const PrefillParams& p, uint32_t s, uint32_t j, uint32_t lane) {
    if (lane >= kBN / 16) return 0;
    const PrefillSeq& sq = p.seq[s];
    const uint64_t npages = ceil_div(sq.kv_tokens, 16);
    const uint64_t lp = static_cast<uint64_t>(j) * (kBN / 16) + lane;
    return __ldg(sq.blocks + (lp < npages ? lp : 0));
}

// One KV tile (8 pages of one KV head) into a ring slot. Warp-wide: page pg's
// id comes from lane pg; the elected lane issues the 16 copies.
__device__ __forceinline__ void load_kv_tile(const PrefillParams& p, const CUtensorMap* map, unsigned char* dst,
                                             uint32_t kh, uint64_t lane_id, bool leader, uint64_t* bar) {
    uint64_t ids[kBN / 16];
#pragma unroll
    for (int pg = 0; pg < kBN / 16; ++pg) ids[pg] = __shfl_sync(0xffffffffu, lane_id, pg);
    if (!leader) return;
    mbar_arrive_expect_tx(bar, kKVTile);
#pragma unroll
    for (int pg = 0; pg < kBN / 16; ++pg) {
        uint64_t blk = ids[pg];
        if (blk >= p.num_blocks) {
            raise_flag(p.status, KVFX_FLAG_BAD_INDEX);
            blk = 0;
        }
#pragma unroll
        for (int b = 0; b < 2; ++b) {
            tma_load_4d(dst + b * kKVHalf + pg * 2048, map, b * 64, 0, static_cast<int>(kh), static_cast<int>(blk),
                        bar);
        }
    }
}

// Producer loop of one ring (K or V) of `kStages` slots, run by a whole warp
// (voted waits, one elected lane issuing the copies): before tile g is
// loaded into slot g % kStages, the MMA that read tile g - kStages must have
// completed, which done[(g - kStages) % nDone] signals (K: k_free, one per
// slot, arrived once QK(g) completes; V: pv_done, the MMA warp's commit once
// PV(g) completes, one per S buffer). Neither barrier can run a phase ahead:
// tile g's own MMA needs this load. The next tile's page ids are fetched
// while waiting for its slot. At the end, waits for its own copies in flight.
__device__ __noinline__ void produce(const PrefillParams& p, const CUtensorMap* map, unsigned char* ring,
                                     uint64_t* full, uint64_t* done, uint32_t kStages, uint32_t nDone) {
    const uint32_t lane = threadIdx.x & 31u;
    const bool leader = elect_one();
    auto wait = [&](uint64_t* bar, uint32_t phase) {
        return __all_sync(0xffffffffu, mbar_wait_lean(bar, phase, p.status)) != 0;
    };
    if (leader) prefetch_tensormap(map);
    TileCursor c;
    c.init(p);
    uint64_t id = c.valid ? tile_page_id(p, c.u.s, c.j, lane) : 0;
    uint32_t issued = 0;
    while (c.valid) {
        const uint32_t g = c.g, st = g % kStages;
        if (g >= kStages) {
            const uint32_t prev = g - kStages;
            if (!wait(&done[prev % nDone], (prev / nDone) & 1u)) break;
        }
        load_kv_tile(p, map, ring + st * kKVTile, c.u.kh, id, leader, &full[st]);
        issued = g + 1;
        c.next(p);
        if (c.valid) id = tile_page_id(p, c.u.s, c.j, lane);
    }
    for (uint32_t g = issued > kStages ? issued - kStages : 0; g < issued; ++g)
        (void)wait(&full[g % kStages], (g / kStages) & 1u);
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
prefill_tc_kernel(const __grid_constant__ PrefillParams p, const __grid_constant__ CUtensorMap kmap,
                  const __grid_constant__ CUtensorMap vmap) {
    extern __shared__ unsigned char smem_raw[];
    __shared__ uint64_t k_full[kKStages], k_free[kKStages], v_full[kVStages];
    __shared__ uint64_t s_full[kSBufs], p_full[kSBufs], pv_done[kSBufs];
    __shared__ uint64_t q_full, q_free, o_full, o_free, mma_done;
    __shared__ uint64_t l_ready[2], l_free[2];
    __shared__ float l_sh[2][kBM];  // row sums of a unit, by unit parity
    __shared__ uint32_t tmem_base_slot;

    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_addr(smem);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (tid == 0) {
        for (int s = 0; s < kKStages; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_free[s], 1);
        }
        for (int s = 0; s < kVStages; ++s) mbar_init(&v_full[s], 1);
        for (int b = 0; b < kSBufs; ++b) {
            mbar_init(&s_full[b], 1);
            mbar_init(&p_full[b], 128);
            mbar_init(&pv_done[b], 1);
        }
        mbar_init(&q_full, 128);
        mbar_init(&q_free, 1);
        mbar_init(&o_full, 1);
        mbar_init(&o_free, 128);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&l_ready[b], 128);
            mbar_init(&l_free[b], 128);
        }
        mbar_init(&mma_done, 1);
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

    if (warp == 0) {
        // ---------------------------------------------------- K producer ---
        produce(p, &kmap, smem + kOffK, k_full, k_free, kKStages, kKStages);
    } else if (warp == 2) {
        // ---------------------------------------------------- V producer ---
        produce(p, &vmap, smem + kOffV, v_full, pv_done, kVStages, kSBufs);
    } else if (warp == 1) {
        // ----------------------------------------------------- MMA issuer ---
        // The whole warp runs the schedule (its values stay warp-uniform);
        // one elected lane issues the MMAs and commits. Waits are voted so
        // that every lane takes the same path.
        {
            const bool leader = elect_one();
            auto wait = [&](uint64_t* bar, uint32_t phase) {
                return __all_sync(0xffffffffu, mbar_wait_lean(bar, phase, p.status)) != 0;
            };
            // Two barriers at once: both try_waits issue back to back and
            // one vote covers them (both are usually complete already); the
            // bounded slow path runs only when one is not.
            auto wait2 = [&](uint64_t* a, uint32_t pa, uint64_t* b, uint32_t pb) {
                const bool fa = mbar_try_wait(smem_addr(a), pa);
                const bool fb = mbar_try_wait(smem_addr(b), pb);
                if (__all_sync(0xffffffffu, fa && fb)) return true;
                return wait(a, pa) && wait(b, pb);
            };
            constexpr bool kBF = std::is_same<T, __nv_bfloat16>::value;
            const uint32_t id_qk = tc::idesc_f16(kBM, kBN, kBF, false);
            const uint32_t id_pv = tc::idesc_f16(kBM, kHD, kBF, true);
            // Operand descriptors are formed once; every MMA adds a constant
            // offset (16-byte units, the descriptor's low start-address field;
            // shared addresses stay below 2^18 so nothing carries out).
            const uint64_t k_desc0 = tc::desc_k_major(sbase + kOffK);
            const uint64_t v_desc0 = tc::desc_mn_major(sbase + kOffV, kKVHalf);
            TileCursor qk, pv;
            qk.init(p);
            pv.init(p);
            // S(g) = Q K_g^T into S[g%2], which held P(g-2): PV(g-2) was
            // issued before this step by this thread and so reads P(g-2)
            // before these MMAs write there. Each step is split into its
            // waits, its 16 MMAs and its commits, so that the next step's
            // waits can run while the tensor pipe still has this step's last
            // MMAs queued.
            auto qk_wait = [&]() -> bool {
                const uint32_t g = qk.g;
                if (qk.j == 0) {
                    if (!wait2(&q_full, qk.k & 1u, &k_full[g % kKStages], (g / kKStages) & 1u)) return false;
                } else if (!wait(&k_full[g % kKStages], (g / kKStages) & 1u)) {
                    return false;
                }
                tc::fence_after_sync();
                return true;
            };
            auto qk_mmas = [&](uint32_t from, uint32_t to) {
                const uint32_t g = qk.g;
                const uint32_t d = tmem + (g % kSBufs) * kBN;
                const uint64_t k_desc = k_desc0 + (((g % kKStages) * kKVTile) >> 4);
                // Q_hi then Q_lo (A from TMEM: 8 columns per 16 dims), 8
                // K-steps of 16 each (unrolled: the constant operand offsets
                // fold into the address and descriptor adds).
#pragma unroll
                for (uint32_t i = 0; i < 16; ++i) {
                    if (i < from || i >= to) continue;
                    const uint32_t part = i >> 3, kk = i & 7;
                    const uint32_t a = tmem + kTmemQ + part * (kHD / 2) + kk * 8;
                    const uint32_t b_off = (kk >> 2) * kKVHalf + (kk & 3) * 32;
                    if (leader) tc::mma_ts(d, a, k_desc + (b_off >> 4), id_qk, i > 0 ? 1u : 0u);
                }
            };
            auto qk_finish = [&]() {
                if (leader) {
                    tc::commit(&s_full[qk.g % kSBufs]);
                    if (qk.last()) tc::commit(&q_free);
                }  // Q may be replaced once this completes
                qk.next(p);
            };
            // O += P(g) V_g with P from TMEM; a unit's first PV overwrites O,
            // which the previous unit's epilogue must have read.
            auto pv_wait = [&]() -> bool {
                const uint32_t g = pv.g;
                if (pv.j == 0 && pv.k >= 1 && !wait(&o_free, (pv.k - 1) & 1u)) return false;
                if (!wait2(&v_full[g % kVStages], (g / kVStages) & 1u, &p_full[g % kSBufs], (g / kSBufs) & 1u))
                    return false;
                tc::fence_after_sync();
                return true;
            };
            auto pv_mmas = [&](uint32_t from, uint32_t to) {
                const uint32_t g = pv.g;
                const uint32_t pt = tmem + (g % kSBufs) * kBN;
                const uint64_t v_desc = v_desc0 + (((g % kVStages) * kKVTile) >> 4);
                // 8 K-steps of 16 tokens, P_hi then P_lo for each.
#pragma unroll
                for (uint32_t i = 0; i < 16; ++i) {
                    if (i < from || i >= to) continue;
                    const uint32_t t = i >> 1, part = i & 1;
                    const uint32_t a = pt + (t >> 1) * 32 + part * 16 + (t & 1) * 8;
                    if (leader)
                        tc::mma_ts(tmem + kTmemO, a, v_desc + ((t * 2048) >> 4), id_pv, (pv.j > 0 || i > 0) ? 1u : 0u);
                }
            };
            auto pv_finish = [&]() {
                if (leader) {
                    tc::commit(&pv_done[pv.g % kSBufs]);
                    if (pv.last()) tc::commit(&o_full);
                }
                pv.next(p);
            };
            constexpr uint32_t kSplit = 12;  // MMAs of a step issued before the next step's waits
            bool ok = true;
            // QK(0), QK(1). Loops here and below keep one copy of each MMA
            // group in the code: the kernel's roles share the SM's
            // instruction cache.
#pragma unroll 1
            for (int i = 0; i < 2 && ok && qk.valid; ++i) {
                ok = qk_wait();
                if (ok) {
                    qk_mmas(0, 16);
                    qk_finish();
                }
            }
            if (ok && pv.valid) ok = pv_wait();
            // Steady state: PV(g), then QK(g + 2).
            while (ok && pv.valid) {
                const bool more_qk = qk.valid;
                // When QK(g + 2) starts a unit, its Q is staged by the warps
                // that also run the epilogue, after the epilogue of the unit
                // before the previous one, which may be waiting for this
                // PV's commit (when the previous unit has one tile): then
                // PV(g) is issued and committed before that wait.
                const bool unit_start = more_qk && qk.j == 0;
                pv_mmas(0, kSplit);
                if (more_qk && !unit_start) ok = qk_wait();
                pv_mmas(kSplit, 16);
                pv_finish();
                if (unit_start) ok = qk_wait();
                if (!ok) break;
                if (more_qk) {
                    // All of QK(g + 2) and its commit before the wait for
                    // P(g + 1): the softmax of tile g + 2 starts as soon as
                    // it is done with g + 1, and 16 queued MMAs cover the wait.
                    qk_mmas(0, 16);
                    qk_finish();
                    if (pv.valid) ok = pv_wait();
                } else if (pv.valid) {
                    ok = pv_wait();
                }
            }
            // Every MMA this thread issued is complete before TMEM is released.
            if (leader) tc::commit(&mma_done);
            (void)wait(&mma_done, 0);
        }
    } else if (warp >= 4 && warp < 8) {
        // -------------------------------------------------------- softmax ---
        const uint32_t quarter = static_cast<uint32_t>(warp & 3);  // TMEM lanes this warp may access
        const uint32_t r = quarter * 32 + lane;                     // query row within the unit
        const uint32_t lane_base = (quarter * 32) << 16;
        const uint32_t tO = tmem + kTmemO + lane_base;
        // tcgen05.ld/st are warp-collective: every wait result is made
        // warp-uniform so that no lane skips one the others execute.
        auto wait_all = [&](uint64_t* bar, uint32_t phase) {
            return __all_sync(0xffffffffu, mbar_wait_lean(bar, phase, p.status)) != 0;
        };
        bool ok = true;
        uint32_t g = 0;  // running tile ordinal, as in the MMA thread
        Unit u;
        for (uint32_t round = 0, k = 0; ok && unit_at(p, round, u); ++round, ++k) {
            // Last visible position of this row.
            const PrefillSeq& sq = p.seq[u.s];
            const int64_t pos = static_cast<int64_t>(sq.kv_tokens - sq.q_tokens + u.q0 + r);
            float m_run = -INFINITY, l_run = 0.f;
            for (uint32_t j = 0; j < u.ntiles; ++j, ++g) {
                const uint32_t b = g % kSBufs;
                if (!wait_all(&s_full[b], (g / kSBufs) & 1u)) { ok = false; break; }
                tc::fence_after_sync();
                // QK(g) has completed, so it has read K tile g: free its slot.
                if (warp == 4 && lane == 0) mbar_arrive(&k_free[g % kKStages]);
                const uint32_t tS = tmem + b * kBN + lane_base;
                // Causal mask: column c is visible iff j*128 + c <= pos (pos <
                // kv_tokens for live rows). Applied as a select against the
                // column's compile-time index, so that masked columns become
                // -inf whatever they held (NaN included); only tiles on or
                // past the diagonal need it.
                const int64_t lim64 = pos - static_cast<int64_t>(j) * kBN;
                const int lim = lim64 < -1 ? -1 : (lim64 > kBN ? kBN : static_cast<int>(lim64));
                const bool masked = !__all_sync(0xffffffffu, lim >= kBN - 1);
                auto mask32 = [&](float* v, int rel) {  // rel: lim relative to v[0]
#pragma unroll
                    for (int cc = 0; cc < 32; ++cc) v[cc] = cc <= rel ? v[cc] : -INFINITY;
                };
                auto max32 = [](const float* v) {
                    float m[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) m[e] = fmax3(v[e], v[4 + e], v[8 + e]);
#pragma unroll
                    for (int q = 12; q < 28; q += 8) {
#pragma unroll
                        for (int e = 0; e < 4; ++e) m[e] = fmax3(m[e], v[q + e], v[q + 4 + e]);
                    }
#pragma unroll
                    for (int e = 0; e < 4; ++e) m[e] = fmaxf(m[e], v[28 + e]);
                    return fmaxf(fmax3(m[0], m[1], m[2]), m[3]);
                };
                // Row maximum: all 128 scores in one TMEM round trip, masked on
                // diagonal tiles.
                float mx;
                {
                    float sc[kBN];
#pragma unroll
                    for (int cb = 0; cb < kBN; cb += 32) tc::ld32(tS + cb, sc + cb);
                    tc::wait_ld32(sc);
                    tc::reg_fence32(sc + 32);
                    tc::reg_fence32(sc + 64);
                    tc::reg_fence32(sc + 96);
                    if (masked) {
#pragma unroll
                        for (int cb = 0; cb < kBN; cb += 32) mask32(sc + cb, lim - cb);
                    }
                    mx = fmaxf(fmaxf(max32(sc), max32(sc + 32)), fmaxf(max32(sc + 64), max32(sc + 96)));
                }
                const bool need = mx > m_run + 8.f;  // m_run = -inf: always at a unit's first tile
                const float m_new = need ? mx : m_run;
                const float alpha = ex2_approx(m_run - m_new);  // 1 if unchanged, 0 at the first tile
                if (j >= 1 && __any_sync(0xffffffffu, need)) {
                    // O holds P(0..j-1) V once PV(g-1) completes; PV(g) is
                    // not issued before this tile's P is published.
                    if (!wait_all(&pv_done[(g - 1) % kSBufs], ((g - 1) / kSBufs) & 1u)) { ok = false; break; }
                    tc::fence_after_sync();
#pragma unroll 1
                    for (int cb = 0; cb < kHD; cb += 32) {
                        float ov[32];
                        tc::ld32(tO + cb, ov);
                        tc::wait_ld32(ov);
#pragma unroll
                        for (int e = 0; e < 32; ++e) ov[e] *= alpha;
                        tc::st32(tO + cb, ov);
                    }
                }
                m_run = m_new;
                // P = exp2(S - m) as packed hi/lo pairs over the tile's own S
                // columns: chunk c (tokens 32c..32c+31) -> hi at 32c, lo at
                // 32c + 16. The scores are read again from TMEM chunk by
                // chunk, the next chunk's load overlapping this chunk's math.
                const uint64_t mm = f2_pack(m_run, m_run);
                uint64_t lsum0 = f2_pack(0.f, 0.f), lsum1 = lsum0;
                auto p_chunk = [&](int c, float* v) {
                    if (masked) mask32(v, lim - 32 * c);
                    // All 16 pairs of the chunk, then its hi and lo halves in
                    // one 16-column store each.
                    uint32_t hi[16], lo[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        float x0, x1;
                        f2_unpack(f2_sub(f2_pack(v[2 * e], v[2 * e + 1]), mm), x0, x1);
                        x0 = ex2_approx(x0);
                        x1 = ex2_approx(x1);
                        const uint64_t pe = f2_pack(x0, x1);
                        if (e & 1) lsum1 = f2_add(lsum1, pe);
                        else lsum0 = f2_add(lsum0, pe);
                        hi[e] = Elem<T>::pack(x0, x1);
                        float r0, r1;
                        f2_unpack(f2_sub(pe, widen2<T>(hi[e])), r0, r1);
                        lo[e] = Elem<T>::pack(r0, r1);
                    }
                    tc::st16(tS + 32 * c, hi);
                    tc::st16(tS + 32 * c + 16, lo);
                };
                {
                    float va[32], vb[32];
                    tc::ld32(tS, va);
                    tc::wait_ld32(va);
#pragma unroll 1
                    for (int c = 0; c < kBN / 32; c += 2) {
                        tc::ld32(tS + 32 * (c + 1), vb);
                        p_chunk(c, va);
                        tc::wait_ld32(vb);
                        if (c + 2 < kBN / 32) tc::ld32(tS + 32 * (c + 2), va);
                        p_chunk(c + 1, vb);
                        if (c + 2 < kBN / 32) tc::wait_ld32(va);
                    }
                }
                {
                    float s0, s1, s2, s3;
                    f2_unpack(lsum0, s0, s1);
                    f2_unpack(lsum1, s2, s3);
                    l_run = l_run * alpha + ((s0 + s1) + (s2 + s3));
                }
                tc::wait_st();
                // Tokens past the sequence end in this tile: zero their V rows
                // (unwritten slots may hold NaN; 0 * NaN must not reach O).
                // Done before P(g) is published, which precedes PV(g).
                const uint64_t t0 = static_cast<uint64_t>(j) * kBN;
                if (t0 + kBN > sq.kv_tokens) {
                    const uint32_t sv = g % kVStages;
                    if (!wait_all(&v_full[sv], (g / kVStages) & 1u)) { ok = false; break; }
                    const uint32_t valid = static_cast<uint32_t>(sq.kv_tokens - t0);
                    const uint32_t rows = kBN - valid;
                    unsigned char* vt = smem + kOffV + sv * kKVTile;
                    for (uint32_t i = r; i < rows * 2 * 8; i += 128) {
                        const uint32_t row = valid + i / 16, half = (i / 8) & 1, cc = i & 7;
                        *reinterpret_cast<uint4*>(vt + half * kKVHalf + row * 128 + cc * 16) =
                            make_uint4(0, 0, 0, 0);
                    }
                    fence_proxy_async_smem();
                }
                tc::fence_before_sync();
                mbar_arrive(&p_full[b]);
            }
            if (!ok) break;
            // Hand the unit's row sums to the epilogue warps (the buffer of
            // this parity was last read for unit k - 2).
            if (k >= 2 && !wait_all(&l_free[k & 1u], ((k - 2) >> 1) & 1u)) break;
            l_sh[k & 1u][r] = l_run;
            mbar_arrive(&l_ready[k & 1u]);
        }
    } else if (warp >= 8) {
        // ------------------------------------------ Q staging + epilogue ---
        // Warp 8 + w accesses TMEM lanes 32w..32w+31 (the quarter its
        // sub-partition may access): row r = its thread's query row.
        // tcgen05.ld/st are warp-collective: every wait result is made
        // warp-uniform.
        const uint32_t quarter = static_cast<uint32_t>(warp & 3);
        const uint32_t r = quarter * 32 + lane;
        const uint32_t lane_base = (quarter * 32) << 16;
        const uint32_t tQ = tmem + kTmemQ + lane_base;
        const uint32_t tO = tmem + kTmemO + lane_base;
        auto wait_all = [&](uint64_t* bar, uint32_t phase) {
            return __all_sync(0xffffffffu, mbar_wait_lean(bar, phase, p.status)) != 0;
        };
        // Row r of unit u's Q (zeros past the sequence's queries).
        // Rows past the sequence's queries load its last query row instead:
        // their scores, weights and O rows stay in their own TMEM lanes and
        // are never stored (and no branch duplicates the load code).
        auto load_q = [&](const Unit& u, float* v) {
            const PrefillSeq& sq = p.seq[u.s];
            const uint64_t qi = umin64(u.q0 + r, sq.q_tokens - 1);
            const float4* qrow = reinterpret_cast<const float4*>(sq.q + (qi * p.q_heads + u.qh) * kHD);
#pragma unroll
            for (int e = 0; e < kHD / 4; ++e) {
                const float4 x = __ldg(qrow + e);
                v[4 * e] = x.x;
                v[4 * e + 1] = x.y;
                v[4 * e + 2] = x.z;
                v[4 * e + 3] = x.w;
            }
        };
        // Scaled hi/lo halves into the Q columns (column c of the hi (lo)
        // half holds dims 2c, 2c+1), then publish.
        const uint64_t qs2 = f2_pack(p.qscale, p.qscale);
        auto write_q = [&](const float* v) {
#pragma unroll
            for (uint32_t cc = 0; cc < kHD / 16; ++cc) {
                uint32_t hi[8], lo[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    // Packed f32x2 arithmetic: the same split as split2_fast.
                    const uint64_t x = f2_mul(f2_pack(v[16 * cc + 2 * e], v[16 * cc + 2 * e + 1]), qs2);
                    float x0, x1;
                    f2_unpack(x, x0, x1);
                    hi[e] = Elem<T>::pack(x0, x1);
                    float r0, r1;
                    f2_unpack(f2_sub(x, widen2<T>(hi[e])), r0, r1);
                    lo[e] = Elem<T>::pack(r0, r1);
                }
                tc::st8(tQ + cc * 8, hi);
                tc::st8(tQ + kHD / 2 + cc * 8, lo);
            }
            tc::wait_st();
            tc::fence_before_sync();
            mbar_arrive(&q_full);
        };
        // Epilogue of unit k (u): O from TMEM, released to the next unit's
        // first PV as soon as it is in registers, then O / l to global
        // memory. Uses v as its buffer.
        float v[kHD];
        auto epilogue = [&](uint32_t k, const Unit& u) -> bool {
            if (!wait_all(&l_ready[k & 1u], (k >> 1) & 1u)) return false;
            if (!wait_all(&o_full, k & 1u)) return false;
            tc::fence_after_sync();
#pragma unroll
            for (int cb = 0; cb < kHD; cb += 32) tc::ld32(tO + cb, v + cb);
            tc::wait_ld32(v);
            tc::reg_fence32(v + 32);
            tc::reg_fence32(v + 64);
            tc::reg_fence32(v + 96);
            tc::fence_before_sync();
            mbar_arrive(&o_free);
            const float inv = 1.f / l_sh[k & 1u][r];
            mbar_arrive(&l_free[k & 1u]);
            const PrefillSeq& sq = p.seq[u.s];
            const uint64_t qi = u.q0 + r;
            if (qi < sq.q_tokens) {
                float4* orow = reinterpret_cast<float4*>(sq.o + (qi * p.q_heads + u.qh) * kHD);
#pragma unroll
                for (int e = 0; e < kHD / 4; ++e)
                    orow[e] = make_float4(v[4 * e] * inv, v[4 * e + 1] * inv, v[4 * e + 2] * inv,
                                          v[4 * e + 3] * inv);
            }
            return true;
        };
        // One pass per unit k: Q(k) into TMEM (the columns are free for the
        // first unit, else once unit k - 1's last QK has read them), then
        // the epilogue of unit k - 1, then the loads of Q(k + 1). One call
        // site each keeps the code small (the roles share the SM's
        // instruction cache).
        Unit cur, nxt, prev;
        uint32_t round = 0;
        bool have = unit_at(p, round, cur);
        if (have) load_q(cur, v);
#pragma unroll 1
        for (uint32_t k = 0;; ++k) {
            if (have) {
                if (k >= 1 && !wait_all(&q_free, (k - 1) & 1u)) break;
                tc::fence_after_sync();
                write_q(v);
            }
            if (k >= 1 && !epilogue(k - 1, prev)) break;
            if (!have) break;
            prev = cur;
            uint32_t nround = round + 1;
            have = unit_at(p, nround, nxt);
            if (have) {
                load_q(nxt, v);
                cur = nxt;
                round = nround;
            }
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
           ceil_div(a.query_tokens, kBM) * a.q_heads < (1ull << 26);  // a launch's units stay below 2^31
}

}  // namespace

bool prefill_tc_supported(const CacheView& c, const AttentionArgs& a) { return prefill_eligible(c, a); }

cudaError_t launch_prefill_tc_batch(const CacheView& c, const AttentionArgs* seqs, uint32_t n, unsigned* status,
                                    cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    if (n > kMaxPrefillSeqs) return cudaErrorInvalidValue;
    cudaError_t err = cudaSuccess;
    const CacheMaps* maps = cache_maps(c, &err);
    if (maps == nullptr) return err != cudaSuccess ? err : cudaErrorInvalidValue;
    static std::atomic<int> attr_done[64];  // zero-initialised; callers on several threads set the same attribute
    const bool bf = c.dtype == KVFX_BF16;
    if (c.device < 0 || c.device >= 64 || !attr_done[c.device].load(std::memory_order_acquire)) {
        err = cudaFuncSetAttribute(prefill_tc_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   kSmemAlloc);
        if (err != cudaSuccess) return err;
        err = cudaFuncSetAttribute(prefill_tc_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   kSmemAlloc);
        if (err != cudaSuccess) return err;
        if (c.device >= 0 && c.device < 64) attr_done[c.device].store(1, std::memory_order_release);
    }
    const int sms = device_sm_count(c.device);
    if (sms <= 0) return cudaErrorInvalidDevice;
    PrefillParams p{};
    uint64_t max_qtiles = 0;
    for (uint32_t i = 0; i < n; ++i) {
        p.seq[i] = PrefillSeq{seqs[i].q, seqs[i].o, seqs[i].blocks, seqs[i].query_tokens, seqs[i].kv_tokens};
        max_qtiles = std::max<uint64_t>(max_qtiles, ceil_div(seqs[i].query_tokens, kBM));
    }
    p.num_seqs = n;
    p.num_blocks = c.num_blocks;
    p.q_heads = seqs[0].q_heads;
    p.kv_heads = c.heads;
    p.group = p.q_heads / c.heads;
    const uint64_t n_units = max_qtiles * n * p.q_heads;
    if (n_units >= (1ull << 31)) return cudaErrorInvalidValue;  // each sequence is checked below 2^26
    p.n_units = static_cast<uint32_t>(n_units);
    p.div_round = make_fastdiv(n * p.q_heads);
    p.div_qheads = make_fastdiv(p.q_heads);
    p.div_group = make_fastdiv(p.group);
    p.qscale = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(c.hd)));
    p.status = status;
    const unsigned grid = static_cast<unsigned>(umin64(p.n_units, static_cast<uint64_t>(sms)));
    if (bf) {
        prefill_tc_kernel<__nv_bfloat16><<<grid, kThreads, kSmemAlloc, s>>>(p, maps->k, maps->v);
    } else {
        prefill_tc_kernel<__half><<<grid, kThreads, kSmemAlloc, s>>>(p, maps->k, maps->v);
    }
    return cudaGetLastError();
}

cudaError_t launch_prefill_tc(const CacheView& c, const AttentionArgs& a, unsigned* status, cudaStream_t s) {
    return launch_prefill_tc_batch(c, &a, 1, status, s);
}

}  // namespace kvfx
