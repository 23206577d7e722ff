/*
 * kvoracle.c - CPU restatement of KVFlux's v2 paged-KV path (see kvoracle.h).
 * TEST INFRASTRUCTURE ONLY: used by tests/, the smoke check and bench.py's
 * CPU baseline as the checker, never by the product.
 *
 * Build: python oracle/build.py  (gcc -O2, no fast-math: FP64 semantics kept).
 */
#include "kvoracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------ helpers --- */

static int mul_ok(uint64_t a, uint64_t b, uint64_t* out) {
    if (b != 0 && a > UINT64_MAX / b) return 0;
    *out = a * b;
    return 1;
}

static float bf16_to_f32(uint16_t h) {
    uint32_t bits = (uint32_t)h << 16;
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

/* IEEE binary16 -> binary32, exact (normals, subnormals, inf, nan). */
static float f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    const uint32_t exp = (h >> 10) & 0x1f;
    const uint32_t man = h & 0x3ff;
    uint32_t bits;
    if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (man << 13);
    } else if (exp != 0) {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    } else if (man == 0) {
        bits = sign;
    } else {
        /* subnormal: value = man * 2^-24, renormalise */
        uint32_t m = man;
        int e = -14;
        while ((m & 0x400u) == 0) {
            m <<= 1;
            --e;
        }
        bits = sign | ((uint32_t)(e + 127) << 23) | ((m & 0x3ffu) << 13);
    }
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

void kvo_to_f32(const void* src, int dtype, uint64_t count, float* dst) {
    uint64_t i;
    if (dtype == 2) {
        memcpy(dst, src, count * sizeof(float));
    } else if (dtype == 1) {
        const uint16_t* s = (const uint16_t*)src;
        for (i = 0; i < count; ++i) dst[i] = bf16_to_f32(s[i]);
    } else {
        const uint16_t* s = (const uint16_t*)src;
        for (i = 0; i < count; ++i) dst[i] = f16_to_f32(s[i]);
    }
}

/* ------------------------------------------------------- write / gather --- */

int kvo_write(uint8_t* k_cache, uint8_t* v_cache, uint64_t num_blocks, uint32_t heads, uint32_t bs,
              uint64_t row_bytes, const uint8_t* k_new, const uint8_t* v_new, const uint64_t* slots,
              uint64_t n) {
    uint64_t i, h, slot_count;
    if (!mul_ok(num_blocks, bs, &slot_count)) return KVO_EOVERFLOW;
    for (i = 0; i < n; ++i) {
        if (slots[i] >= slot_count) return KVO_ERANGE;
    }
    for (i = 0; i < n; ++i) {
        const uint64_t page = slots[i] / bs, off = slots[i] % bs;
        for (h = 0; h < heads; ++h) {
            const uint64_t dst = ((page * heads + h) * bs + off) * row_bytes;
            const uint64_t src = (i * heads + h) * row_bytes;
            memcpy(k_cache + dst, k_new + src, row_bytes);
            memcpy(v_cache + dst, v_new + src, row_bytes);
        }
    }
    return KVO_OK;
}

int kvo_gather(const uint8_t* k_cache, const uint8_t* v_cache, uint64_t num_blocks, uint32_t heads,
               uint32_t bs, uint64_t row_bytes, const uint64_t* blocks, uint64_t num_tokens,
               uint8_t* k_out, uint8_t* v_out) {
    uint64_t t, h;
    for (t = 0; t < num_tokens; ++t) {
        const uint64_t page = blocks[t / bs];
        if (page >= num_blocks) return KVO_ERANGE;
        for (h = 0; h < heads; ++h) {
            const uint64_t src = ((page * heads + h) * bs + t % bs) * row_bytes;
            const uint64_t dst = (t * heads + h) * row_bytes;
            memcpy(k_out + dst, k_cache + src, row_bytes);
            memcpy(v_out + dst, v_cache + src, row_bytes);
        }
    }
    return KVO_OK;
}

/* ------------------------------------------------------ reference math --- */

/* One query token, all heads: the body of the reference's q_token loop
 * (src/v2/reference_attention.cpp:54-88). `scores` has room for kv_tokens. */
static void attend_token(const float* q, const float* k, const float* v, uint64_t q_token,
                         uint64_t q_tokens, uint64_t kv_tokens, uint64_t q_heads, uint64_t kv_heads,
                         uint64_t hd, double scale, double* scores, float* out) {
    const uint64_t last_visible = kv_tokens - q_tokens + q_token;
    const uint64_t per_kv = q_heads / kv_heads;
    uint64_t qh, kt, d;
    for (qh = 0; qh < q_heads; ++qh) {
        const uint64_t kh = qh / per_kv;
        const uint64_t q_off = (q_token * q_heads + qh) * hd;
        double maximum = -INFINITY;
        for (kt = 0; kt <= last_visible; ++kt) {
            const uint64_t k_off = (kt * kv_heads + kh) * hd;
            double dot = 0.0;
            for (d = 0; d < hd; ++d) dot += (double)q[q_off + d] * k[k_off + d];
            scores[kt] = dot * scale;
            if (scores[kt] > maximum) maximum = scores[kt];
        }
        double denominator = 0.0;
        for (kt = 0; kt <= last_visible; ++kt) {
            scores[kt] = exp(scores[kt] - maximum);
            denominator += scores[kt];
        }
        for (d = 0; d < hd; ++d) {
            double result = 0.0;
            for (kt = 0; kt <= last_visible; ++kt) {
                const uint64_t v_off = (kt * kv_heads + kh) * hd;
                result += (scores[kt] / denominator) * v[v_off + d];
            }
            out[q_off + d] = (float)result;
        }
    }
}

int kvo_reference_attention(const float* q, const float* k, const float* v, uint64_t q_tokens,
                            uint64_t kv_tokens, uint64_t q_heads, uint64_t kv_heads, uint64_t head_size,
                            float* out) {
    uint64_t q_elems, kv_elems, tmp, i;
    if (q_heads == 0 || kv_heads == 0 || head_size == 0 || q_heads % kv_heads != 0 ||
        q_tokens > kv_tokens) {
        return KVO_EINVAL;
    }
    if (!mul_ok(q_tokens, q_heads, &tmp) || !mul_ok(tmp, head_size, &q_elems)) return KVO_EOVERFLOW;
    if (!mul_ok(kv_tokens, kv_heads, &tmp) || !mul_ok(tmp, head_size, &kv_elems)) return KVO_EOVERFLOW;
    for (i = 0; i < q_elems; ++i) if (!isfinite(q[i])) return KVO_EINVAL;
    for (i = 0; i < kv_elems; ++i) if (!isfinite(k[i]) || !isfinite(v[i])) return KVO_EINVAL;
    for (i = 0; i < q_elems; ++i) out[i] = 0.0f;
    if (q_tokens == 0) return KVO_OK;
    {
        const double scale = 1.0 / sqrt((double)head_size);
        double* scores = (double*)malloc(sizeof(double) * (size_t)kv_tokens);
        uint64_t qt;
        if (scores == NULL) return KVO_EOVERFLOW;
        for (qt = 0; qt < q_tokens; ++qt) {
            attend_token(q, k, v, qt, q_tokens, kv_tokens, q_heads, kv_heads, head_size, scale, scores, out);
        }
        free(scores);
    }
    return KVO_OK;
}

/* ---------------------------------------------------- threaded drivers --- */

typedef struct {
    const uint8_t* k_cache;
    const uint8_t* v_cache;
    int dtype;
    uint64_t num_blocks;
    uint32_t kv_heads, bs, hd, q_heads;
    const uint64_t* table;
    uint64_t max_blocks;
    const uint64_t* lens;
    const float* q;
    float* out;
    /* decode: items are requests; rows: items are query tokens of one sequence */
    uint64_t item_begin, item_end, stride;
    uint64_t q_tokens, kv_tokens; /* rows mode */
    int mode;                     /* 0 decode, 1 rows */
    int status;
} Job;

static int gather_f32(const Job* j, const uint64_t* blocks, uint64_t len, float* kf, float* vf,
                      uint8_t* scratch_k, uint8_t* scratch_v) {
    const uint64_t elem = j->dtype == 2 ? 4 : 2;
    const uint64_t row_bytes = (uint64_t)j->hd * elem;
    const int rc = kvo_gather(j->k_cache, j->v_cache, j->num_blocks, j->kv_heads, j->bs, row_bytes, blocks,
                              len, scratch_k, scratch_v);
    if (rc != KVO_OK) return rc;
    kvo_to_f32(scratch_k, j->dtype, len * j->kv_heads * j->hd, kf);
    kvo_to_f32(scratch_v, j->dtype, len * j->kv_heads * j->hd, vf);
    return KVO_OK;
}

static void* run_job(void* arg) {
    Job* j = (Job*)arg;
    const uint64_t elem = j->dtype == 2 ? 4 : 2;
    uint64_t it;
    uint64_t cap = 0;
    float *kf = NULL, *vf = NULL;
    uint8_t *sk = NULL, *sv = NULL;
    double* scores = NULL;
    j->status = KVO_OK;
    if (j->mode == 1) {
        cap = j->kv_tokens;
        kf = (float*)malloc(sizeof(float) * cap * j->kv_heads * j->hd);
        vf = (float*)malloc(sizeof(float) * cap * j->kv_heads * j->hd);
        sk = (uint8_t*)malloc(cap * j->kv_heads * j->hd * elem);
        sv = (uint8_t*)malloc(cap * j->kv_heads * j->hd * elem);
        scores = (double*)malloc(sizeof(double) * cap);
        if (!kf || !vf || !sk || !sv || !scores) {
            j->status = KVO_EOVERFLOW;
            goto done;
        }
        j->status = gather_f32(j, j->table, j->kv_tokens, kf, vf, sk, sv);
        if (j->status != KVO_OK) goto done;
    }
    for (it = j->item_begin; it < j->item_end; it += j->stride) {
        if (j->mode == 0) {
            const uint64_t len = j->lens[it];
            const double scale = 1.0 / sqrt((double)j->hd);
            if (len > cap) {
                free(kf); free(vf); free(sk); free(sv); free(scores);
                cap = len;
                kf = (float*)malloc(sizeof(float) * cap * j->kv_heads * j->hd);
                vf = (float*)malloc(sizeof(float) * cap * j->kv_heads * j->hd);
                sk = (uint8_t*)malloc(cap * j->kv_heads * j->hd * elem);
                sv = (uint8_t*)malloc(cap * j->kv_heads * j->hd * elem);
                scores = (double*)malloc(sizeof(double) * cap);
                if (!kf || !vf || !sk || !sv || !scores) {
                    j->status = KVO_EOVERFLOW;
                    goto done;
                }
            }
            if (len == 0) { j->status = KVO_EINVAL; goto done; }
            j->status = gather_f32(j, j->table + it * j->max_blocks, len, kf, vf, sk, sv);
            if (j->status != KVO_OK) goto done;
            /* one query at the last position: q_tokens = 1, kv_tokens = len */
            attend_token(j->q + it * j->q_heads * j->hd, kf, vf, 0, 1, len, j->q_heads, j->kv_heads, j->hd,
                         scale, scores, j->out + it * j->q_heads * j->hd);
        } else {
            const double scale = 1.0 / sqrt((double)j->hd);
            attend_token(j->q, kf, vf, it, j->q_tokens, j->kv_tokens, j->q_heads, j->kv_heads, j->hd, scale,
                         scores, j->out);
        }
    }
done:
    free(kf); free(vf); free(sk); free(sv); free(scores);
    return NULL;
}

static int run_jobs(Job* proto, uint64_t begin, uint64_t end, int threads) {
    int t, rc = KVO_OK;
    Job* jobs;
    pthread_t* tids;
    if (threads < 1) threads = 1;
    if ((uint64_t)threads > end - begin) threads = (int)(end - begin);
    if (threads < 1) return KVO_OK;
    jobs = (Job*)calloc((size_t)threads, sizeof(Job));
    tids = (pthread_t*)calloc((size_t)threads, sizeof(pthread_t));
    if (!jobs || !tids) { free(jobs); free(tids); return KVO_EOVERFLOW; }
    for (t = 0; t < threads; ++t) {
        jobs[t] = *proto;
        jobs[t].item_begin = begin + (uint64_t)t;
        jobs[t].item_end = end;
        jobs[t].stride = (uint64_t)threads;
        if (threads == 1) run_job(&jobs[t]);
        else pthread_create(&tids[t], NULL, run_job, &jobs[t]);
    }
    for (t = 0; t < threads; ++t) {
        if (threads > 1) pthread_join(tids[t], NULL);
        if (jobs[t].status != KVO_OK) rc = jobs[t].status;
    }
    free(jobs);
    free(tids);
    return rc;
}

int kvo_decode_batch(const uint8_t* k_cache, const uint8_t* v_cache, int dtype, uint64_t num_blocks,
                     uint32_t kv_heads, uint32_t bs, uint32_t head_size, const uint64_t* table,
                     uint64_t max_blocks, const uint64_t* lens, uint64_t first, uint64_t count,
                     uint32_t q_heads, const float* q, float* out, int threads) {
    Job proto;
    if (kv_heads == 0 || q_heads == 0 || q_heads % kv_heads != 0 || head_size == 0 || bs == 0) return KVO_EINVAL;
    memset(&proto, 0, sizeof proto);
    proto.k_cache = k_cache;
    proto.v_cache = v_cache;
    proto.dtype = dtype;
    proto.num_blocks = num_blocks;
    proto.kv_heads = kv_heads;
    proto.bs = bs;
    proto.hd = head_size;
    proto.q_heads = q_heads;
    proto.table = table;
    proto.max_blocks = max_blocks;
    proto.lens = lens;
    proto.q = q;
    proto.out = out;
    proto.mode = 0;
    return run_jobs(&proto, first, first + count, threads);
}

int kvo_attention_rows(const uint8_t* k_cache, const uint8_t* v_cache, int dtype, uint64_t num_blocks,
                       uint32_t kv_heads, uint32_t bs, uint32_t head_size, const uint64_t* blocks,
                       uint64_t q_tokens, uint64_t kv_tokens, uint32_t q_heads, const float* q,
                       uint64_t row_begin, uint64_t row_end, float* out, int threads) {
    Job proto;
    if (kv_heads == 0 || q_heads == 0 || q_heads % kv_heads != 0 || head_size == 0 || bs == 0 ||
        q_tokens > kv_tokens || row_end > q_tokens || row_begin > row_end) {
        return KVO_EINVAL;
    }
    memset(&proto, 0, sizeof proto);
    proto.k_cache = k_cache;
    proto.v_cache = v_cache;
    proto.dtype = dtype;
    proto.num_blocks = num_blocks;
    proto.kv_heads = kv_heads;
    proto.bs = bs;
    proto.hd = head_size;
    proto.q_heads = q_heads;
    proto.table = blocks;
    proto.q = q;
    proto.out = out;
    proto.q_tokens = q_tokens;
    proto.kv_tokens = kv_tokens;
    proto.mode = 1;
    return run_jobs(&proto, row_begin, row_end, threads);
}
