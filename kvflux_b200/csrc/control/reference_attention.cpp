// Host-side reference attention: the CPU correctness check that KVFlux ships
// in its library (reference: src/v2/reference_attention.cpp:28-91, declared in
// include/kvflux/v2/reference_attention.h). No GPU entry point of this library
// calls it; it exists so that programs written against KVFlux's API (its own
// tests among them) link and can compare the GPU kernels with it.
//
// Semantics kept: shape checks and their exception types in the reference's
// order, FP64 accumulation, scores scaled by 1/sqrt(head_size), the row max
// subtracted before exp, a causal window that ends at kv_tokens -
// query_tokens + i for query i, output (sum_t (e_t / denominator) * v_t) in
// token order. Arrangement here: one pass computes each row's normalised
// weights once, and V is then walked row by row (contiguous head_size runs)
// with every output dimension accumulated in token order, so each output
// element sees the same sequence of FP64 operations as the reference's
// dimension-major loop and the results are bit-identical.
#include "kvflux/v2/reference_attention.h"

#include <cmath>
#include <limits>
#include <stdexcept>

namespace kvflux::v2 {
namespace {

std::size_t product(std::size_t a, std::size_t b) {
    if (b != 0 && a > std::numeric_limits<std::size_t>::max() / b) {
        throw std::overflow_error("reference attention tensor size overflow");
    }
    return a * b;
}

bool all_finite(const std::vector<float>& xs) {
    for (const float x : xs) {
        if (!std::isfinite(x)) return false;
    }
    return true;
}

}  // namespace

std::vector<float> reference_attention(const std::vector<float>& query, const std::vector<float>& key,
                                       const std::vector<float>& value, const AttentionShape& shape) {
    const std::size_t lq = shape.query_tokens, lkv = shape.kv_tokens;
    const std::size_t hq = shape.query_heads, hkv = shape.kv_heads, hd = shape.head_size;
    if (hq == 0 || hkv == 0 || hd == 0 || hq % hkv != 0 || lq > lkv) {
        throw std::invalid_argument("invalid reference attention shape");
    }
    const std::size_t q_elems = product(product(lq, hq), hd);
    const std::size_t kv_elems = product(product(lkv, hkv), hd);
    if (query.size() != q_elems || key.size() != kv_elems || value.size() != kv_elems) {
        throw std::invalid_argument("reference attention tensor size does not match shape");
    }
    if (!all_finite(query) || !all_finite(key) || !all_finite(value)) {
        throw std::invalid_argument("reference attention inputs must be finite");
    }
    std::vector<float> out(q_elems, 0.0f);
    if (lq == 0) return out;

    const double scale = 1.0 / std::sqrt(static_cast<double>(hd));
    const std::size_t group = hq / hkv;
    const std::size_t kv_row = hkv * hd;  // elements between one token's rows
    std::vector<double> weight(lkv);
    std::vector<double> acc(hd);
    for (std::size_t i = 0; i < lq; ++i) {
        const std::size_t visible = lkv - lq + i + 1;  // tokens [0, visible)
        for (std::size_t h = 0; h < hq; ++h) {
            const std::size_t kh = h / group;
            const float* qv = query.data() + (i * hq + h) * hd;
            const float* kt = key.data() + kh * hd;
            double top = -std::numeric_limits<double>::infinity();
            for (std::size_t t = 0; t < visible; ++t, kt += kv_row) {
                double dot = 0.0;
                for (std::size_t d = 0; d < hd; ++d) dot += static_cast<double>(qv[d]) * kt[d];
                const double s = dot * scale;
                weight[t] = s;
                if (s > top) top = s;
            }
            double sum = 0.0;
            for (std::size_t t = 0; t < visible; ++t) {
                weight[t] = std::exp(weight[t] - top);
                sum += weight[t];
            }
            for (std::size_t t = 0; t < visible; ++t) weight[t] /= sum;
            for (std::size_t d = 0; d < hd; ++d) acc[d] = 0.0;
            const float* vt = value.data() + kh * hd;
            for (std::size_t t = 0; t < visible; ++t, vt += kv_row) {
                const double wt = weight[t];
                for (std::size_t d = 0; d < hd; ++d) acc[d] += wt * vt[d];
            }
            float* o = out.data() + (i * hq + h) * hd;
            for (std::size_t d = 0; d < hd; ++d) o[d] = static_cast<float>(acc[d]);
        }
    }
    return out;
}

}  // namespace kvflux::v2
