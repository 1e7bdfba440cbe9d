/*
 * ArcLLM-B200 oracle (TEST INFRASTRUCTURE ONLY): CPU restatement of the
 * reference's decode hot-path arithmetic.  See orc.h for the contract.
 *
 * Build: gcc -std=c11 -O2 -ffp-contract=off -fPIC -shared -pthread orc.c -lm
 * (oracle/build.py).  -ffp-contract=off matters: the reference computes
 * `d*float(sc)*float(q) - dmin*float(mn)` as separately rounded fp32 ops.
 */
#define _GNU_SOURCE
#include "orc.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* src/p8c_segmented_access_correctness.cpp:503-529 (bit-level fp16 -> fp32;
 * NaN payloads are preserved, subnormals are normalised). */
float orc_half_to_float(uint16_t h) {
    uint32_t sign = ((uint32_t)(h & 0x8000u)) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t mant = h & 0x03ffu;
    uint32_t out;
    if (exp == 0) {
        if (mant == 0) {
            out = sign;
        } else {
            int e = -14;
            while ((mant & 0x0400u) == 0) { mant <<= 1; --e; }
            mant &= 0x03ffu;
            out = sign | ((uint32_t)(e + 127) << 23) | (mant << 13);
        }
    } else if (exp == 31) {
        out = sign | 0x7f800000u | (mant << 13);
    } else {
        out = sign | ((exp - 15u + 127u) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &out, sizeof f);
    return f;
}

/* IEEE-754 binary32 -> binary16, round to nearest even (the same rounding as
 * CUDA's __float2half_rn for every finite input; NaN -> 0x7e00). */
uint16_t orc_float_to_half_rne(float f) {
    uint32_t x;
    memcpy(&x, &f, sizeof x);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xffu;
    uint32_t mant = x & 0x7fffffu;
    if (exp == 0xffu) return (uint16_t)(sign | (mant ? 0x7e00u : 0x7c00u));
    int e = (int)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        mant |= 0x800000u;
        int shift = 14 - e;
        uint32_t hm = mant >> shift;
        uint32_t rem = mant & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (hm & 1u))) hm++;
        return (uint16_t)(sign | hm);
    }
    uint32_t hm = mant >> 13;
    uint32_t rem = mant & 0x1fffu;
    uint32_t h = sign | ((uint32_t)e << 10) | hm;
    if (rem > 0x1000u || (rem == 0x1000u && (hm & 1u))) h++;
    return (uint16_t)h;
}

/* src/p8c_segmented_access_correctness.cpp:531-540: unpack the 6-bit scale and
 * min of sub-block j from the 12 packed bytes at block+4. */
void orc_q4k_scale_min(const uint8_t *block, int j, uint8_t *sc, uint8_t *mn) {
    const uint8_t *q = block + 4;
    if (j < 4) {
        *sc = q[j] & 63;
        *mn = q[j + 4] & 63;
    } else {
        *sc = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
        *mn = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

static inline uint16_t ld_u16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* src/p8c_segmented_access_correctness.cpp:1166-1181 (q4k_dequant_row_p8c). */
void orc_q4k_dequant_row(const uint8_t *row, float *y, uint32_t n) {
    uint32_t nb = n / 256u;
    for (uint32_t ib = 0; ib < nb; ++ib) {
        const uint8_t *b = row + (uint64_t)ib * 144u;
        float d = orc_half_to_float(ld_u16(b)), dmin = orc_half_to_float(ld_u16(b + 2));
        for (uint32_t k = 0; k < 256u; ++k) {
            uint8_t sc, mn;
            orc_q4k_scale_min(b, (int)(k >> 5u), &sc, &mn);
            uint32_t g = k >> 6u, l = k & 63u;
            uint8_t qb = b[16u + g * 32u + (l & 31u)];
            uint8_t q = l < 32u ? (qb & 15u) : (qb >> 4u);
            y[ib * 256u + k] = d * (float)sc * (float)q - dmin * (float)mn;
        }
    }
}

/* src/p8c_segmented_access_correctness.cpp:905-926: 6-bit code of element k
 * (minus 32) and its signed sub-block scale. */
int orc_q6k_value(const uint8_t *b, uint32_t k, int *scale) {
    uint32_t half128 = k >> 7u, kk = k & 127u, l = kk & 31u, quarter = kk >> 5u;
    const uint8_t *ql = b + half128 * 64u;
    const uint8_t *qh = b + 128u + half128 * 32u;
    const uint8_t *sc = b + 192u + half128 * 8u;
    uint32_t is = l >> 4u, low, high, sc_idx;
    if (quarter == 0u) {
        low = ql[l] & 15u; high = (qh[l] >> 0u) & 3u; sc_idx = is + 0u;
    } else if (quarter == 1u) {
        low = ql[l + 32u] & 15u; high = (qh[l] >> 2u) & 3u; sc_idx = is + 2u;
    } else if (quarter == 2u) {
        low = ql[l] >> 4u; high = (qh[l] >> 4u) & 3u; sc_idx = is + 4u;
    } else {
        low = ql[l + 32u] >> 4u; high = (qh[l] >> 6u) & 3u; sc_idx = is + 6u;
    }
    uint8_t s = sc[sc_idx];
    *scale = s >= 128u ? (int)s - 256 : (int)s;
    return (int)(low | (high << 4u)) - 32;
}

/* src/p8c_segmented_access_correctness.cpp:944-956. */
void orc_q6k_dequant_row(const uint8_t *row, float *y, uint32_t n) {
    uint32_t nb = n / 256u;
    for (uint32_t ib = 0; ib < nb; ++ib) {
        const uint8_t *b = row + (uint64_t)ib * 210u;
        float d = orc_half_to_float(ld_u16(b + 208));
        for (uint32_t k = 0; k < 256u; ++k) {
            int sc = 0;
            int q = orc_q6k_value(b, k, &sc);
            y[ib * 256u + k] = d * (float)sc * (float)q;
        }
    }
}

/* src/p8c_segmented_access_correctness.cpp:542-567. */
float orc_q4k_dot_row(const uint8_t *row, const float *x, uint32_t n) {
    const uint32_t nblocks = n / 256u;
    float sum = 0.0f;
    for (uint32_t ib = 0; ib < nblocks; ++ib) {
        const uint8_t *b = row + ib * 144u;
        float d = orc_half_to_float(ld_u16(b));
        float dmin = orc_half_to_float(ld_u16(b + 2));
        for (uint32_t k = 0; k < 256u; ++k) {
            uint8_t sc = 0, mn = 0;
            orc_q4k_scale_min(b, (int)(k >> 5u), &sc, &mn);
            uint32_t group64 = k >> 6u, local64 = k & 63u;
            uint8_t qb = b[16u + group64 * 32u + (local64 & 31u)];
            uint8_t q = local64 < 32u ? (qb & 15u) : (qb >> 4u);
            float w = d * (float)sc * (float)q - dmin * (float)mn;
            sum += w * x[ib * 256u + k];
        }
    }
    return sum;
}

/* src/p8c_segmented_access_correctness.cpp:928-942. */
float orc_q6k_dot_row(const uint8_t *row, const float *x, uint32_t n) {
    float sum = 0.0f;
    uint32_t nb = n / 256u;
    for (uint32_t ib = 0; ib < nb; ++ib) {
        const uint8_t *b = row + (uint64_t)ib * 210u;
        float d = orc_half_to_float(ld_u16(b + 208));
        for (uint32_t k = 0; k < 256u; ++k) {
            int sc = 0;
            int q = orc_q6k_value(b, k, &sc);
            sum += (d * (float)sc * (float)q) * x[ib * 256u + k];
        }
    }
    return sum;
}

/* ---- row-parallel matmul (the per-row arithmetic is the reference's) ---- */
typedef struct {
    const uint8_t *w; uint32_t n, rows, batch, r0, r1, q6;
    const float *x, *bias; float *y;
} mm_job;

static void *mm_worker(void *arg) {
    const mm_job *j = (const mm_job *)arg;
    uint64_t rb = (uint64_t)(j->n / 256u) * (j->q6 ? 210u : 144u);
    for (uint32_t b = 0; b < j->batch; ++b) {
        const float *xb = j->x + (uint64_t)b * j->n;
        for (uint32_t r = j->r0; r < j->r1; ++r) {
            const uint8_t *row = j->w + (uint64_t)r * rb;
            float v = j->q6 ? orc_q6k_dot_row(row, xb, j->n) : orc_q4k_dot_row(row, xb, j->n);
            j->y[(uint64_t)b * j->rows + r] = v + (j->bias ? j->bias[r] : 0.0f);
        }
    }
    return NULL;
}

static void matmul_any(const uint8_t *w, uint32_t n, uint32_t rows, uint32_t batch,
                       const float *x, const float *bias, float *y, int threads, int q6) {
    if (threads <= 1 || rows < 2) {
        mm_job j = {w, n, rows, batch, 0, rows, (uint32_t)q6, x, bias, y};
        mm_worker(&j);
        return;
    }
    if ((uint32_t)threads > rows) threads = (int)rows;
    pthread_t *tid = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)threads);
    mm_job *jobs = (mm_job *)malloc(sizeof(mm_job) * (size_t)threads);
    for (int t = 0; t < threads; ++t) {
        uint32_t r0 = (uint32_t)((uint64_t)rows * (uint64_t)t / (uint64_t)threads);
        uint32_t r1 = (uint32_t)((uint64_t)rows * (uint64_t)(t + 1) / (uint64_t)threads);
        mm_job j = {w, n, rows, batch, r0, r1, (uint32_t)q6, x, bias, y};
        jobs[t] = j;
        pthread_create(&tid[t], NULL, mm_worker, &jobs[t]);
    }
    for (int t = 0; t < threads; ++t) pthread_join(tid[t], NULL);
    free(jobs);
    free(tid);
}

/* src/p8c_segmented_access_correctness.cpp:971-984 */
void orc_matmul_q4(const uint8_t *w, uint32_t n, uint32_t rows, uint32_t batch,
                   const float *x, const float *bias, float *y, int threads) {
    matmul_any(w, n, rows, batch, x, bias, y, threads, 0);
}

/* src/p8c_segmented_access_correctness.cpp:986-999 */
void orc_matmul_q6(const uint8_t *w, uint32_t n, uint32_t rows, uint32_t batch,
                   const float *x, const float *bias, float *y, int threads) {
    matmul_any(w, n, rows, batch, x, bias, y, threads, 1);
}

/* src/p8c_segmented_access_correctness.cpp:958-969: double sum of squares,
 * fp32 inverse root, y = x*inv*w. */
void orc_rmsnorm(const float *x, const float *w, uint32_t batch, uint32_t n, float eps, float *y) {
    for (uint32_t b = 0; b < batch; ++b) {
        double ss = 0.0;
        const float *xb = x + (uint64_t)b * n;
        for (uint32_t i = 0; i < n; ++i) ss += (double)xb[i] * (double)xb[i];
        float inv = 1.0f / sqrtf((float)(ss / (double)n) + eps);
        for (uint32_t i = 0; i < n; ++i) y[(uint64_t)b * n + i] = xb[i] * inv * w[i];
    }
}

/* src/p8c_segmented_access_correctness.cpp:1001-1018: adjacent-pair rotation
 * of (x[2p], x[2p+1]) by pos * theta^(-2p/dim). */
void orc_rope(float *x, uint32_t batch, uint32_t heads, uint32_t dim, uint32_t pos_base, float theta) {
    for (uint32_t b = 0; b < batch; ++b) {
        uint32_t pos = pos_base + b;
        for (uint32_t h = 0; h < heads; ++h) {
            uint64_t base = ((uint64_t)b * heads + h) * dim;
            for (uint32_t p = 0; p < dim / 2u; ++p) {
                uint64_t i0 = base + 2u * p, i1 = i0 + 1u;
                float angle = (float)pos * powf(theta, -2.0f * (float)p / (float)dim);
                float c = cosf(angle), s = sinf(angle);
                float a = x[i0], bb = x[i1];
                x[i0] = a * c - bb * s;
                x[i1] = a * s + bb * c;
            }
        }
    }
}

/* src/p8c_segmented_access_correctness.cpp:1064-1073 */
void orc_swiglu(const float *g, const float *u, uint32_t n, float *y) {
    for (uint32_t i = 0; i < n; ++i) {
        float gv = g[i];
        y[i] = (gv / (1.0f + expf(-gv))) * u[i];
    }
}

/* src/p8c_segmented_access_correctness.cpp:1057-1062 */
void orc_add(const float *a, const float *b, uint32_t n, float *y) {
    for (uint32_t i = 0; i < n; ++i) y[i] = a[i] + b[i];
}

/* src/p8c_segmented_access_correctness.cpp:1136-1158: scores in double,
 * rounded to float; float max; exp in float; double normaliser; double
 * weighted sum of V. */
void orc_attention_cache(const float *q, const float *kc, const float *vc,
                         uint32_t layer, uint32_t pos, uint32_t max_ctx,
                         uint32_t q_heads, uint32_t kv_heads, uint32_t dim, float *out) {
    uint32_t heads_per_kv = q_heads / kv_heads;
    float scale = 1.0f / sqrtf((float)dim);
    float *scores = (float *)malloc(sizeof(float) * (pos + 1u));
    for (uint32_t qh = 0; qh < q_heads; ++qh) {
        uint32_t kvh = qh / heads_per_kv;
        float mx = -INFINITY;
        for (uint32_t t = 0; t <= pos; ++t) {
            double s = 0.0;
            uint64_t kb = (((uint64_t)layer * max_ctx + t) * kv_heads + kvh) * dim;
            for (uint32_t d = 0; d < dim; ++d) s += (double)q[(uint64_t)qh * dim + d] * (double)kc[kb + d];
            scores[t] = (float)(s * scale);
            mx = fmaxf(mx, scores[t]);
        }
        double sm = 0.0;
        for (uint32_t t = 0; t <= pos; ++t) { scores[t] = expf(scores[t] - mx); sm += scores[t]; }
        for (uint32_t t = 0; t <= pos; ++t) scores[t] = (float)(scores[t] / sm);
        for (uint32_t d = 0; d < dim; ++d) {
            double a = 0.0;
            for (uint32_t t = 0; t <= pos; ++t) {
                uint64_t vb = (((uint64_t)layer * max_ctx + t) * kv_heads + kvh) * dim + d;
                a += (double)scores[t] * (double)vc[vb];
            }
            out[(uint64_t)qh * dim + d] = (float)a;
        }
    }
    free(scores);
}

/* src/p8c_segmented_access_correctness.cpp:1163 argmax_ptr. */
uint32_t orc_argmax(const float *p, uint32_t n, int *finite) {
    uint32_t bi = 0;
    float bv = p[0];
    int fin = isfinite(bv) ? 1 : 0;
    for (uint32_t i = 1; i < n; ++i) {
        float v = p[i];
        if (!isfinite(v)) fin = 0;
        if (v > bv) { bv = v; bi = i; }
    }
    if (finite) *finite = fin;
    return bi;
}

/* ---- synthetic fixture streams ------------------------------------------ */
/* splitmix64 finaliser; sequence element n of seed s is mix(s + (n+1)*gamma),
 * which is exactly the sequential generator of
 * src/sa1_component_benchmark.cpp:71-76 evaluated at its (n+1)-th call. */
static inline uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint64_t orc_splitmix64_at(uint64_t seed, uint64_t n) {
    return mix64(seed + (n + 1u) * 0x9E3779B97F4A7C15ull);
}

static inline float unit24(uint64_t w) { return (float)(uint32_t)(w >> 40) * 5.9604644775390625e-08f; }

static inline void put16(uint8_t *p, uint16_t v) { p[0] = (uint8_t)(v & 255u); p[1] = (uint8_t)(v >> 8); }

enum { Q4_WORDS = 20, Q6_WORDS = 27 };

void orc_fill_q4k(uint8_t *dst, uint64_t block_begin, uint64_t n_blocks, uint64_t seed) {
    for (uint64_t i = 0; i < n_blocks; ++i) {
        uint64_t blk = block_begin + i, base = blk * Q4_WORDS;
        uint8_t *b = dst + i * 144u;
        uint64_t w[Q4_WORDS];
        for (int k = 0; k < Q4_WORDS; ++k) w[k] = orc_splitmix64_at(seed, base + (uint64_t)k);
        float t = 3e-3f * unit24(w[0]);
        float d = 1e-3f + t;
        float dmin = 2e-3f * unit24(w[1]);
        put16(b, orc_float_to_half_rne(d));
        put16(b + 2, orc_float_to_half_rne(dmin));
        uint8_t v[16];
        for (int j = 0; j < 16; ++j)
            v[j] = (uint8_t)(j < 10 ? (w[2] >> (6 * j)) & 63u : (w[3] >> (6 * (j - 10))) & 63u);
        const uint8_t *sc = v, *mn = v + 8;
        uint8_t *q = b + 4;
        for (int j = 0; j < 4; ++j) {
            q[j] = (uint8_t)((sc[j] & 63u) | ((sc[j + 4] >> 4) << 6));
            q[j + 4] = (uint8_t)((mn[j] & 63u) | ((mn[j + 4] >> 4) << 6));
        }
        for (int j = 4; j < 8; ++j) q[j + 4] = (uint8_t)((sc[j] & 15u) | ((mn[j] & 15u) << 4));
        for (int k = 0; k < 128; ++k) b[16 + k] = (uint8_t)(w[4 + k / 8] >> (8 * (k % 8)));
    }
}

void orc_fill_q6k(uint8_t *dst, uint64_t block_begin, uint64_t n_blocks, uint64_t seed) {
    for (uint64_t i = 0; i < n_blocks; ++i) {
        uint64_t blk = block_begin + i, base = blk * Q6_WORDS;
        uint8_t *b = dst + i * 210u;
        uint64_t w[Q6_WORDS];
        for (int k = 0; k < Q6_WORDS; ++k) w[k] = orc_splitmix64_at(seed, base + (uint64_t)k);
        for (int k = 0; k < 192; ++k) b[k] = (uint8_t)(w[k / 8] >> (8 * (k % 8)));
        for (int j = 0; j < 16; ++j) {
            uint32_t v = (uint32_t)(j < 10 ? (w[24] >> (6 * j)) & 63u : (w[25] >> (6 * (j - 10))) & 63u);
            b[192 + j] = (uint8_t)(int8_t)((int)v - 32);
        }
        float t = 3e-3f * unit24(w[26]);
        put16(b + 208, orc_float_to_half_rne(1e-3f + t));
    }
}

static inline float ih_normal(uint64_t w, float mu, float sigma) {
    int32_t s = (int32_t)((w & 0xffffu) + ((w >> 16) & 0xffffu) + ((w >> 32) & 0xffffu) + (w >> 48));
    float z = (float)(s - 131070) * (1.7320508075688772f * 1.52587890625e-05f);
    float t = sigma * z;
    return mu + t;
}

void orc_fill_normal_f32(float *dst, uint64_t begin, uint64_t n, uint64_t seed, float mu, float sigma) {
    for (uint64_t i = 0; i < n; ++i) dst[i] = ih_normal(orc_splitmix64_at(seed, begin + i), mu, sigma);
}

void orc_fill_normal_f16(uint16_t *dst, uint64_t begin, uint64_t n, uint64_t seed, float mu, float sigma) {
    for (uint64_t i = 0; i < n; ++i)
        dst[i] = orc_float_to_half_rne(ih_normal(orc_splitmix64_at(seed, begin + i), mu, sigma));
}

void orc_fill_tokens(uint32_t *dst, uint64_t n, uint64_t seed, uint32_t vocab) {
    for (uint64_t i = 0; i < n; ++i)
        dst[i] = (uint32_t)(((orc_splitmix64_at(seed, i) >> 32) * (uint64_t)vocab) >> 32);
}
