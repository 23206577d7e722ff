// Device-side helpers shared by the sm_100a kernels: element types, the
// status word, bounded waits, and thin inline-PTX wrappers for mbarrier,
// bulk/tensor TMA loads, ldmatrix and mma.sync.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kvfx.h"
#include "launch.h"

namespace kvfx {

// --------------------------------------------------------------- division ---

// n / d for n < 2^31 with one multiply-high: m = floor(2^32 (2^s - d) / d) + 1,
// s = ceil(log2 d) (the round-up multiplier of Granlund and Montgomery, 1994).
struct FastDiv {
    uint32_t m, s;
};

inline FastDiv make_fastdiv(uint32_t d) {
    uint32_t s = 0;
    while ((1ull << s) < d) ++s;
    const uint64_t m = ((1ull << 32) * ((1ull << s) - d)) / d + 1;
    return FastDiv{static_cast<uint32_t>(m), s};
}

__device__ __forceinline__ uint32_t fast_div(uint32_t n, FastDiv f) { return (__umulhi(n, f.m) + n) >> f.s; }

// ---------------------------------------------------------------- status ---

// Set bits of the per-device status word (mapped host memory, or a
// __device__ word for callers that pass one of their own).
__device__ __forceinline__ void raise_flag(unsigned* status, unsigned bit) {
    if (status != nullptr) atomicOr(status, bit);
}

// Programmatic dependent launch. A kernel launched with the programmatic
// stream-serialization attribute may be scheduled before the kernel ahead of
// it on the stream has finished; pdl_wait() then blocks until that kernel has
// completed and its memory writes are visible (a no-op for a kernel launched
// without the attribute), so it must precede the first global memory access.
// pdl_allow_next() lets the stream's next such kernel be scheduled early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_allow_next() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Upper bound of any device-side wait: generous against the longest
// legitimate wait (a TMA load of a few KiB), short enough to return control.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// -------------------------------------------------------------- mbarrier ---

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbarrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                 ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar_addr, uint32_t phase) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done) : "r"(bar_addr), "r"(phase) : "memory");
    return done != 0;
}

// Waits for the phase with parity `phase` to complete. Returns false (and
// raises KVFX_FLAG_TIMEOUT) if it has not completed within kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t phase, unsigned* status) {
    const uint32_t a = smem_addr(bar);
    if (mbar_try_wait(a, phase)) return true;
    const uint64_t start = globaltimer_ns();
    for (uint32_t spin = 0;; ++spin) {
        if (mbar_try_wait(a, phase)) return true;
        if ((spin & 63u) == 63u) {
            if (globaltimer_ns() - start > kWaitLimitNs) {
                raise_flag(status, KVFX_FLAG_TIMEOUT);
                return false;
            }
            __nanosleep(64);
        }
    }
}

// Slow part of mbar_wait_lean, kept out of line so that each call site adds
// only one try_wait to the caller's code (for kernels whose hot loops must
// stay small in the instruction cache).
static __device__ __noinline__ bool mbar_wait_slow(uint32_t a, uint32_t phase, unsigned* status) {
    const uint64_t start = globaltimer_ns();
    for (uint32_t spin = 0;; ++spin) {
        if (mbar_try_wait(a, phase)) return true;
        if ((spin & 15u) == 15u) {
            if (globaltimer_ns() - start > kWaitLimitNs) {
                raise_flag(status, KVFX_FLAG_TIMEOUT);
                return false;
            }
            __nanosleep(32);
        }
    }
}

// Same contract as mbar_wait.
__device__ __forceinline__ bool mbar_wait_lean(uint64_t* bar, uint32_t phase, unsigned* status) {
    const uint32_t a = smem_addr(bar);
    if (mbar_try_wait(a, phase)) return true;
    return mbar_wait_slow(a, phase, status);
}

// True in exactly one lane of a converged warp (PTX elect.sync): code that
// one thread must issue (tensor-core MMAs, commits) runs under it while the
// whole warp computes its operands, which stay warp-uniform.
__device__ __forceinline__ bool elect_one() {
    uint32_t is = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(is));
    return is != 0;
}

// ---------------------------------------------------------- bulk copies ---

// 1-D bulk copy global -> shared, completion counted on `bar` (bytes % 16 == 0,
// both addresses 16-byte aligned).
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                         uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_addr(smem_dst)), "l"(gmem_src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// Tiled 4-D tensor load (no multicast) into shared memory, completion on `bar`.
__device__ __forceinline__ void tma_load_4d(void* smem_dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, int c3, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6];"
        ::"r"(smem_addr(smem_dst)), "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
          "r"(smem_addr(bar))
        : "memory");
}

// Tiled 3-D tensor store from shared memory, tracked as a bulk-async group:
// commit with bulk_commit(), then bulk_wait_read<N>() returns once all but
// the N most recent groups have finished reading shared memory, and
// bulk_wait<N>() once they have completed.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, int c0, int c1, int c2, const void* smem_src) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%1, %2, %3}], [%4];"
                 ::"l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(smem_addr(smem_src))
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait() {
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ------------------------------------------------------------ tensor ops ---

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

template <typename T> struct MmaKind;
template <> struct MmaKind<__nv_bfloat16> {
    static __device__ __forceinline__ void mma(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
            "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
};
template <> struct MmaKind<__half> {
    static __device__ __forceinline__ void mma(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
            "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
};

// ---------------------------------------------------------- conversions ---

template <typename T> struct Elem;
template <> struct Elem<float> {
    static __device__ __forceinline__ float to_f32(float x) { return x; }
};
template <> struct Elem<__half> {
    static __device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
    static __device__ __forceinline__ __half from_f32(float x) { return __float2half_rn(x); }
    // Packs two floats (lo in the low half) after round-to-nearest.
    static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
        __half2 h = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&h);
    }
};
template <> struct Elem<__nv_bfloat16> {
    static __device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
    static __device__ __forceinline__ __nv_bfloat16 from_f32(float x) { return __float2bfloat16_rn(x); }
    static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
        __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&h);
    }
};

// 2^x by the MUFU approximation (flush-to-zero; 2^-inf = +0).
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// max(a, b, c) in one instruction (sm_100 three-input form).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// Two floats in one 64-bit register pair, for the sm_100 packed f32x2 ops.
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t x, float& a, float& b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(x));
}
__device__ __forceinline__ uint64_t f2_add(uint64_t x, uint64_t y) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(x), "l"(y));
    return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t x, uint64_t y) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(x), "l"(y));
    return r;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t x, uint64_t y) {
    uint64_t r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(x), "l"(y));
    return r;
}

// Same split as split2 below with one rounding per pair: the packed hi is
// widened back by bit moves (bf16) or conversions (fp16) instead of a
// second round of the already representable values.
template <typename T>
__device__ __forceinline__ void split2_fast(float x0, float x1, uint32_t& hi, uint32_t& lo);
template <>
__device__ __forceinline__ void split2_fast<__nv_bfloat16>(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    hi = Elem<__nv_bfloat16>::pack(x0, x1);
    const float h0 = __uint_as_float(hi << 16), h1 = __uint_as_float(hi & 0xFFFF0000u);
    lo = Elem<__nv_bfloat16>::pack(x0 - h0, x1 - h1);
}
template <>
__device__ __forceinline__ void split2_fast<__half>(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    hi = Elem<__half>::pack(x0, x1);
    const __half2 h = *reinterpret_cast<const __half2*>(&hi);
    lo = Elem<__half>::pack(x0 - __low2float(h), x1 - __high2float(h));
}

// Splits x into hi + lo, both representable in T, with hi = round(x) and
// lo = round(x - hi); hi + lo carries about twice T's mantissa bits.
template <typename T>
__device__ __forceinline__ void split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    const T h0 = Elem<T>::from_f32(x0), h1 = Elem<T>::from_f32(x1);
    hi = Elem<T>::pack(Elem<T>::to_f32(h0), Elem<T>::to_f32(h1));
    lo = Elem<T>::pack(x0 - Elem<T>::to_f32(h0), x1 - Elem<T>::to_f32(h1));
}

}  // namespace kvfx
