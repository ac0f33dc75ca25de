/*
 * weaver_oracle.c — CPU oracle for the Weaver decode attention.
 *
 * TEST INFRASTRUCTURE ONLY (see weaver_oracle.h).  Compiled with
 * -ffp-contract=off so that every multiply and add rounds separately, as the
 * scalar reference loops are written.
 */
#include "weaver_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORACLE_BLOCK 16u          /* ModelDims::BLOCK_SIZE, types.rs:159 */
#define ORACLE_K 4u               /* ModelDims::SPARSITY_K, types.rs:160 */
#define ORACLE_REF_MASK 0x7FFFFFFFu /* weaver_kernel.metal:145,174 */

/* ------------------------------------------------------------------------- */
/* binary16 conversions                                                      */
/* ------------------------------------------------------------------------- */

float oracle_h2f(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t m = h & 0x3FFu;
    uint32_t bits;
    float f;
    if (e == 0) {
        /* zero or subnormal: m * 2^-24, exact in binary32 */
        f = (float)m * 5.9604644775390625e-8f;
        return sign ? -f : f;
    }
    if (e == 31) bits = sign | 0x7F800000u | (m << 13);
    else bits = sign | ((e + 112u) << 23) | (m << 13);
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t oracle_f2h(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) { /* inf / nan (nan stays quiet, payload truncated) */
        if (ax == 0x7F800000u) return sign | 0x7C00u;
        return (uint16_t)(sign | 0x7E00u | ((ax >> 13) & 0x3FFu));
    }
    if (ax < 0x38800000u) { /* below 2^-14: binary16 subnormal or zero */
        float v;
        memcpy(&v, &ax, 4);
        /* v * 2^24 is exact; nearbyintf rounds half to even in the default mode */
        uint32_t q = (uint32_t)nearbyintf(v * 16777216.0f);
        return (uint16_t)(sign | q); /* q == 1024 is the smallest normal, bits agree */
    }
    uint32_t e = (ax >> 23) - 112u;
    uint32_t mant = ax & 0x7FFFFFu;
    uint32_t h = (e << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    if (h >= 0x7C00u) h = 0x7C00u; /* overflow rounds to infinity */
    return (uint16_t)(sign | h);
}

/* ------------------------------------------------------------------------- */
/* Literal restatement of weaver_kernel.metal:118-240                        */
/* ------------------------------------------------------------------------- */

/* simd_reduce_add (weaver_kernel.metal:58-66): butterfly over 32 lanes with
 * xor distances 16, 8, 4, 2, 1.  All lanes end with the same value. */
static float lanes_reduce_add(float v[32]) {
    static const unsigned masks[5] = {16, 8, 4, 2, 1};
    float t[32];
    for (int s = 0; s < 5; ++s) {
        for (unsigned l = 0; l < 32; ++l) t[l] = v[l] + v[l ^ masks[s]];
        memcpy(v, t, sizeof(t));
    }
    return v[0];
}

int oracle_literal_decode(const uint16_t* q_exact, const uint16_t* q_latent,
                          const uint16_t* hot_pool, uint64_t hot_pool_blocks,
                          const oracle_sparse_code* cold_pool, uint64_t cold_pool_blocks,
                          const uint32_t* loom_refs, const uint16_t* dictionary,
                          const oracle_weaver_params* p, uint16_t* out) {
    const uint32_t d = p->head_dim;   /* the reference hard-codes 128 (:23) */
    const uint32_t A = p->dict_size;  /* the reference hard-codes 512 (:26) */
    const uint32_t Hkv = p->kv_heads;
    const uint32_t B = ORACLE_BLOCK;
    if (d == 0 || d > 256 || p->gqa_group == 0 || Hkv == 0) return -2;
    const uint32_t chunk = (d + 31) / 32; /* head_dim_chunk (:134) */

    for (uint32_t head = 0; head < p->q_heads; ++head) {
        const uint32_t kv_head = head / p->gqa_group; /* :131 */
        if (kv_head >= Hkv) return -2;
        float m = -INFINITY, l = 0.0f;
        float acc[32][8]; /* acc[lane][i] holds dim lane + 32*i */
        memset(acc, 0, sizeof(acc));

        /* Pass 1: hot segment (:143-168) */
        for (uint32_t b = 0; b < p->hot_count; ++b) {
            const uint32_t phys = loom_refs[b] & ORACLE_REF_MASK;
            if ((uint64_t)phys >= hot_pool_blocks) return -1;
            for (uint32_t t = 0; t < B; ++t) {
                const uint64_t k_off = (uint64_t)phys * B * Hkv * d + (uint64_t)t * Hkv * d +
                                       (uint64_t)kv_head * d;
                float part[32];
                for (uint32_t lane = 0; lane < 32; ++lane) {
                    float s = 0.0f;
                    for (uint32_t i = lane; i < d; i += 32)
                        s += oracle_h2f(q_exact[(uint64_t)head * d + i]) *
                             oracle_h2f(hot_pool[k_off + i]);
                    part[lane] = s;
                }
                const float score = lanes_reduce_add(part);
                /* online_softmax_update (:69-96), V row = K row (:163) */
                const float new_m = fmaxf(m, score);
                const float exp_old = expf(m - new_m);
                const float exp_new = expf(score - new_m);
                for (uint32_t lane = 0; lane < 32; ++lane)
                    for (uint32_t i = 0; i < chunk; ++i) acc[lane][i] *= exp_old;
                l = l * exp_old + exp_new;
                m = new_m;
                for (uint32_t lane = 0; lane < 32; ++lane)
                    for (uint32_t i = 0; i < chunk; ++i) {
                        const uint32_t idx = lane + i * 32;
                        if (idx < d) acc[lane][i] += exp_new * oracle_h2f(hot_pool[k_off + idx]);
                    }
            }
        }

        /* Pass 2: cold segment (:172-222) */
        for (uint32_t b = 0; b < p->cold_count; ++b) {
            const uint32_t phys = loom_refs[p->hot_count + b] & ORACLE_REF_MASK;
            if ((uint64_t)phys >= cold_pool_blocks) return -1;
            for (uint32_t t = 0; t < B; ++t) {
                const uint64_t code_idx = (uint64_t)phys * B * Hkv + (uint64_t)t * Hkv + kv_head;
                const oracle_sparse_code code = cold_pool[code_idx];
                float score = 0.0f;
                for (uint32_t k = 0; k < ORACLE_K; ++k) {
                    if (code.indices[k] >= A) return -1;
                    score += oracle_h2f(q_latent[(uint64_t)head * A + code.indices[k]]) *
                             oracle_h2f(code.coeffs[k]);
                }
                const float new_m = fmaxf(m, score);
                const float exp_old = expf(m - new_m);
                const float exp_new = expf(score - new_m);
                for (uint32_t lane = 0; lane < 32; ++lane)
                    for (uint32_t i = 0; i < chunk; ++i) acc[lane][i] *= exp_old;
                l = l * exp_old + exp_new;
                m = new_m;
                for (uint32_t lane = 0; lane < 32; ++lane)
                    for (uint32_t i = 0; i < chunk; ++i) {
                        const uint32_t dim = lane + i * 32;
                        if (dim < d) {
                            float v = 0.0f;
                            for (uint32_t k = 0; k < ORACLE_K; ++k) {
                                const uint64_t di = (uint64_t)kv_head * A * d +
                                                    (uint64_t)code.indices[k] * d + dim;
                                v += oracle_h2f(code.coeffs[k]) * oracle_h2f(dictionary[di]);
                            }
                            acc[lane][i] += exp_new * v;
                        }
                    }
            }
        }

        /* Finalize (:226-239) */
        for (uint32_t lane = 0; lane < 32; ++lane)
            for (uint32_t i = 0; i < chunk; ++i) {
                const uint32_t dim = lane + i * 32;
                if (dim >= d) continue;
                float a = acc[lane][i];
                if (l > 0.0f) a /= l;
                out[(uint64_t)head * d + dim] = oracle_f2h(a);
            }
    }
    return 0;
}

/* ------------------------------------------------------------------------- */
/* Configuration mode                                                        */
/* ------------------------------------------------------------------------- */

static int check_desc(const oracle_decode_desc* d) {
    if (!d->q || !d->hot_k || !d->hot_v || !d->hot_refs || !d->hot_indptr) return -2;
    if (!d->cold_refs || !d->cold_indptr || !d->k_codes || !d->v_codes) return -2;
    if (!d->v_dict || (!d->k_dict && !d->q_latent)) return -2;
    if (d->kv_heads == 0 || d->q_heads % d->kv_heads) return -2;
    if (d->head_dim == 0 || d->dict_size == 0 || d->num_queries == 0) return -2;
    return 0;
}

/* One query row (b, j, h), generic over the accumulation type. */
#define DEFINE_ROW(NAME, T, EXP)                                                              \
    static int NAME(const oracle_decode_desc* D, uint32_t b, uint32_t j, uint32_t h, T* acc, \
                    T* qlat) {                                                               \
        const uint32_t d = D->head_dim, A = D->dict_size, Hkv = D->kv_heads;                 \
        const uint32_t G = D->q_heads / Hkv, g = h / G, nq = D->num_queries;                 \
        const uint64_t row = ((uint64_t)b * nq + j) * D->q_heads + h;                        \
        const uint16_t* qv = D->q + row * d;                                                 \
        const uint16_t* kd = D->k_dict ? D->k_dict + (uint64_t)g * D->dict_head_stride : 0;  \
        const uint16_t* vd = D->v_dict + (uint64_t)g * D->dict_head_stride;                  \
        /* q_latent (absent in the reference, weaver.rs:142): q . K_dict per atom */         \
        for (uint32_t a = 0; a < A; ++a) {                                                   \
            if (D->q_latent) {                                                               \
                qlat[a] = (T)oracle_h2f(D->q_latent[row * A + a]);                           \
            } else {                                                                         \
                T s = 0;                                                                     \
                for (uint32_t i = 0; i < d; ++i)                                             \
                    s += (T)oracle_h2f(qv[i]) * (T)oracle_h2f(kd[(uint64_t)a * d + i]);      \
                qlat[a] = s * (T)D->scale;                                                   \
            }                                                                                \
        }                                                                                    \
        for (uint32_t i = 0; i < d; ++i) acc[i] = 0;                                         \
        T m = -INFINITY, l = 0;                                                              \
        const uint32_t h0 = D->hot_indptr[b], h1 = D->hot_indptr[b + 1];                     \
        const uint64_t Th = (uint64_t)(h1 - h0) * ORACLE_BLOCK;                              \
        uint64_t limit = Th;                                                                 \
        if (D->causal) { /* ops.metal:549 applied to the hot tail */                         \
            if (Th + 1 < nq) return -2;                                                      \
            limit = Th - nq + 1 + j;                                                         \
        }                                                                                    \
        for (uint32_t pb = h0; pb < h1; ++pb) {                                              \
            const uint32_t phys = D->hot_refs[pb] & ORACLE_REF_MASK;                         \
            if ((uint64_t)phys >= D->hot_pool_blocks) return -1;                             \
            for (uint32_t t = 0; t < ORACLE_BLOCK; ++t) {                                    \
                const uint64_t pos = (uint64_t)(pb - h0) * ORACLE_BLOCK + t;                 \
                if (pos >= limit) continue;                                                  \
                const uint64_t off = (((uint64_t)phys * ORACLE_BLOCK + t) * Hkv + g) * d;    \
                T s = 0;                                                                     \
                for (uint32_t i = 0; i < d; ++i)                                             \
                    s += (T)oracle_h2f(qv[i]) * (T)oracle_h2f(D->hot_k[off + i]);            \
                s *= (T)D->scale;                                                            \
                const T nm = s > m ? s : m;                                                  \
                const T eo = EXP(m - nm), en = EXP(s - nm);                                  \
                for (uint32_t i = 0; i < d; ++i)                                             \
                    acc[i] = acc[i] * eo + en * (T)oracle_h2f(D->hot_v[off + i]);            \
                l = l * eo + en;                                                             \
                m = nm;                                                                      \
            }                                                                                \
        }                                                                                    \
        const uint32_t c0 = D->cold_indptr[b], c1 = D->cold_indptr[b + 1];                   \
        for (uint32_t pb = c0; pb < c1; ++pb) {                                              \
            const uint32_t phys = D->cold_refs[pb] & ORACLE_REF_MASK;                        \
            if ((uint64_t)phys >= D->cold_pool_blocks) return -1;                            \
            for (uint32_t t = 0; t < ORACLE_BLOCK; ++t) {                                    \
                const uint64_t ci = ((uint64_t)phys * ORACLE_BLOCK + t) * Hkv + g;           \
                const oracle_sparse_code kc = D->k_codes[ci], vc = D->v_codes[ci];           \
                T s = 0;                                                                     \
                for (uint32_t k = 0; k < ORACLE_K; ++k) {                                    \
                    if (kc.indices[k] >= A || vc.indices[k] >= A) return -1;                 \
                    s += (T)oracle_h2f(kc.coeffs[k]) * qlat[kc.indices[k]];                  \
                }                                                                            \
                const T nm = s > m ? s : m;                                                  \
                const T eo = EXP(m - nm), en = EXP(s - nm);                                  \
                for (uint32_t i = 0; i < d; ++i) {                                           \
                    T v = 0;                                                                 \
                    for (uint32_t k = 0; k < ORACLE_K; ++k)                                  \
                        v += (T)oracle_h2f(vc.coeffs[k]) *                                   \
                             (T)oracle_h2f(vd[(uint64_t)vc.indices[k] * d + i]);             \
                    acc[i] = acc[i] * eo + en * v;                                           \
                }                                                                            \
                l = l * eo + en;                                                             \
                m = nm;                                                                      \
            }                                                                                \
        }                                                                                    \
        if (D->out) {                                                                        \
            for (uint32_t i = 0; i < d; ++i)                                                 \
                D->out[row * d + i] = oracle_f2h((float)(l > 0 ? acc[i] / l : 0));           \
        }                                                                                    \
        if (D->out_m) D->out_m[row] = (float)m;                                              \
        if (D->out_l) D->out_l[row] = (float)l;                                              \
        if (D->out_o)                                                                        \
            for (uint32_t i = 0; i < d; ++i) D->out_o[row * d + i] = (float)acc[i];          \
        return 0;                                                                            \
    }

DEFINE_ROW(row_f64, double, exp)
DEFINE_ROW(row_f32, float, expf)

int oracle_config_decode_f64(const oracle_decode_desc* D) {
    if (check_desc(D)) return -2;
    double* acc = (double*)malloc(sizeof(double) * D->head_dim);
    double* qlat = (double*)malloc(sizeof(double) * D->dict_size);
    int rc = (acc && qlat) ? 0 : -3;
    for (uint32_t b = 0; b < D->num_seqs && !rc; ++b)
        for (uint32_t j = 0; j < D->num_queries && !rc; ++j)
            for (uint32_t h = 0; h < D->q_heads && !rc; ++h) rc = row_f64(D, b, j, h, acc, qlat);
    free(acc);
    free(qlat);
    return rc;
}

int oracle_config_decode_f32(const oracle_decode_desc* D, int threads) {
    if (check_desc(D)) return -2;
    const int64_t rows = (int64_t)D->num_seqs * D->num_queries * D->q_heads;
    int rc = 0;
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel num_threads(threads) reduction(min : rc)
#endif
    {
        float* acc = (float*)malloc(sizeof(float) * D->head_dim);
        float* qlat = (float*)malloc(sizeof(float) * D->dict_size);
        if (!acc || !qlat) rc = -3;
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int64_t r = 0; r < rows; ++r) {
            if (!acc || !qlat) continue;
            const uint32_t h = (uint32_t)(r % D->q_heads);
            const uint32_t j = (uint32_t)((r / D->q_heads) % D->num_queries);
            const uint32_t b = (uint32_t)(r / ((int64_t)D->q_heads * D->num_queries));
            const int e = row_f32(D, b, j, h, acc, qlat);
            if (e < rc) rc = e;
        }
        free(acc);
        free(qlat);
    }
    (void)threads;
    return rc;
}

/* ------------------------------------------------------------------------- */
/* Atom selection (distiller.rs:185-234)                                     */
/* ------------------------------------------------------------------------- */

/* Ranking: higher score first; NaN after every number; equal scores by
 * ascending atom index. */
static int ranks_before(float sa, uint32_t ia, float sb, uint32_t ib) {
    const int na = isnan(sa), nb = isnan(sb);
    if (na != nb) return nb; /* the non-NaN one ranks first */
    if (!na && sa != sb) return sa > sb;
    return ia < ib;
}

int oracle_distill_rows(const uint16_t* rows, uint32_t n_rows, uint32_t kv_heads,
                        uint32_t head_dim, const uint16_t* dict, uint32_t dict_size,
                        uint64_t dict_head_stride, oracle_sparse_code* out) {
    if (kv_heads == 0 || head_dim == 0) return -2;
    for (uint32_t r = 0; r < n_rows; ++r) {
        const uint16_t* x = rows + (uint64_t)r * head_dim;
        const uint32_t g = r % kv_heads;
        const uint16_t* D = dict + (uint64_t)g * dict_head_stride;
        float best_s[ORACLE_K];
        uint32_t best_i[ORACLE_K];
        uint32_t nbest = 0;
        for (uint32_t a = 0; a < dict_size; ++a) {
            /* f32 dot summed in order from -0.0 (Rust's <f32 as Sum>); each
             * f16*f16 product is exact in binary32 */
            float s = -0.0f;
            for (uint32_t i = 0; i < head_dim; ++i)
                s += oracle_h2f(x[i]) * oracle_h2f(D[(uint64_t)a * head_dim + i]);
            /* insertion into the running top-4 */
            uint32_t pos = nbest;
            while (pos > 0 && ranks_before(s, a, best_s[pos - 1], best_i[pos - 1])) --pos;
            if (pos < ORACLE_K) {
                uint32_t last = nbest < ORACLE_K ? nbest : ORACLE_K - 1;
                for (uint32_t q = last; q > pos; --q) {
                    best_s[q] = best_s[q - 1];
                    best_i[q] = best_i[q - 1];
                }
                best_s[pos] = s;
                best_i[pos] = a;
                if (nbest < ORACLE_K) ++nbest;
            }
        }
        oracle_sparse_code c;
        memset(&c, 0, sizeof(c));
        for (uint32_t k = 0; k < nbest; ++k) {
            c.indices[k] = (uint16_t)best_i[k];
            c.coeffs[k] = oracle_f2h(best_s[k]);
        }
        out[r] = c;
    }
    return 0;
}

float oracle_block_entropy(const uint16_t* values, uint64_t n) {
    if (n == 0) return 0.0f;
    int all_zero = 1;
    for (uint64_t i = 0; i < n && all_zero; ++i)
        if (oracle_h2f(values[i]) != 0.0f) all_zero = 0;
    if (all_zero) return 0.0f;
    double sum = 0.0;
    for (uint64_t i = 0; i < n; ++i) sum += (double)oracle_h2f(values[i]);
    const double mean = sum / (double)n;
    double var = 0.0;
    for (uint64_t i = 0; i < n; ++i) {
        const double diff = (double)oracle_h2f(values[i]) - mean;
        var += diff * diff;
    }
    return (float)(var / (double)n);
}

/* ops.metal:528-616.  One threadgroup per (query head, query token) of
 * tgs = min(64, d) threads (ops.rs:456-459); thread t takes positions t,
 * t + tgs, ...  Phase order and reductions as the kernel's: scores (fp32, sum
 * over dimensions in order from 0, times 1/sqrt(d)); per-thread maxima, then
 * shared[t] = max(shared[t], shared[t + s]) for s = tgs/2, tgs/4, ..., 1;
 * exp(score - max) with per-thread partial sums reduced the same way; every
 * score divided by the sum; output dimension d = sum over positions in order
 * of p[pos] * V[pos][d], cast to f16. */
int oracle_mha(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, uint16_t* out,
               uint32_t total_kv_len, uint32_t head_dim, uint32_t q_heads, uint32_t kv_heads,
               uint32_t num_queries) {
    if (head_dim == 0 || kv_heads == 0 || q_heads % kv_heads || total_kv_len < num_queries) return -2;
    const uint32_t tgs = head_dim < 64 ? head_dim : 64;
    const uint32_t G = q_heads / kv_heads, kv_stride = kv_heads * head_dim;
    const float scale = 1.0f / sqrtf((float)head_dim);
    float* scores = (float*)malloc(sizeof(float) * (total_kv_len ? total_kv_len : 1));
    float shared[64];
    if (!scores) return -3;
    for (uint32_t qi = 0; qi < num_queries; ++qi) {
        const uint32_t valid = total_kv_len - num_queries + 1 + qi;
        for (uint32_t h = 0; h < q_heads; ++h) {
            const uint32_t g = h / G;
            const uint16_t* Q = q + ((uint64_t)qi * q_heads + h) * head_dim;
            uint16_t* O = out + ((uint64_t)qi * q_heads + h) * head_dim;
            for (uint32_t pos = 0; pos < valid; ++pos) {
                const uint16_t* K = k_cache + (uint64_t)pos * kv_stride + (uint64_t)g * head_dim;
                float sc = 0.0f;
                for (uint32_t i = 0; i < head_dim; ++i) sc += oracle_h2f(Q[i]) * oracle_h2f(K[i]);
                scores[pos] = sc * scale;
            }
            for (uint32_t t = 0; t < tgs; ++t) {
                float m = -INFINITY;
                for (uint32_t pos = t; pos < valid; pos += tgs) m = (m < scores[pos]) ? scores[pos] : m;
                shared[t] = m;
            }
            for (uint32_t st = tgs / 2; st > 0; st >>= 1)
                for (uint32_t t = 0; t < st; ++t) shared[t] = (shared[t] < shared[t + st]) ? shared[t + st] : shared[t];
            const float gmax = shared[0];
            for (uint32_t t = 0; t < tgs; ++t) {
                float sum = 0.0f;
                for (uint32_t pos = t; pos < valid; pos += tgs) {
                    scores[pos] = expf(scores[pos] - gmax);
                    sum += scores[pos];
                }
                shared[t] = sum;
            }
            for (uint32_t st = tgs / 2; st > 0; st >>= 1)
                for (uint32_t t = 0; t < st; ++t) shared[t] += shared[t + st];
            const float total = shared[0];
            for (uint32_t pos = 0; pos < valid; ++pos) scores[pos] /= total;
            for (uint32_t d = 0; d < head_dim; ++d) {
                float acc = 0.0f;
                for (uint32_t pos = 0; pos < valid; ++pos)
                    acc += scores[pos] * oracle_h2f(v_cache[(uint64_t)pos * kv_stride + (uint64_t)g * head_dim + d]);
                O[d] = oracle_f2h(acc);
            }
        }
    }
    free(scores);
    return 0;
}
