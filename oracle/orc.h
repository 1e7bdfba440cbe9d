/*
 * ArcLLM-B200 oracle: a plain-C CPU restatement of ArcLLM's decode hot-path
 * arithmetic.  TEST INFRASTRUCTURE ONLY -- this library is the checker used by
 * tests/, __graft_entry__.smoke() and the cpu_baseline leg of bench.py.  The
 * product path (arcllm_b200/libarcllm_cuda.so) never links or calls it.
 *
 * Every function cites the reference function it restates (paths are relative
 * to the ArcLLM repository root).  Arithmetic order follows the reference
 * exactly: fp32 sequential accumulation, no FMA contraction (the library is
 * compiled with -ffp-contract=off), double accumulation where the reference
 * uses double.
 *
 * Parity pin: tests/test_oracle_golden.py checks every function below against
 * golden vectors produced by the reference's own code (oracle/_ref, compiled in
 * place from src/p8c_segmented_access_correctness.cpp and the header-only
 * src/q6cb_q6_reference.hpp, src/q4_down_exec148_materializer.h).
 */
#ifndef ARCLLM_ORACLE_ORC_H
#define ARCLLM_ORACLE_ORC_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- fp16 <-> fp32 ---------------------------------------------------- */
float    orc_half_to_float(uint16_t h);                 /* p8c:503-529 */
uint16_t orc_float_to_half_rne(float f);                /* IEEE-754 RNE (fixture packing) */

/* ---- super-block decode (bit-exact dequant) ---------------------------- */
void orc_q4k_scale_min(const uint8_t *block, int j, uint8_t *sc, uint8_t *mn); /* p8c:531-540 */
void orc_q4k_dequant_row(const uint8_t *row, float *y, uint32_t n);            /* p8c:1166-1181 */
int  orc_q6k_value(const uint8_t *block, uint32_t k, int *scale);             /* p8c:905-926 */
void orc_q6k_dequant_row(const uint8_t *row, float *y, uint32_t n);            /* p8c:944-956 */

/* ---- matvec (sequential fp32, reference order) -------------------------- */
float orc_q4k_dot_row(const uint8_t *row, const float *x, uint32_t n);        /* p8c:542-567 */
float orc_q6k_dot_row(const uint8_t *row, const float *x, uint32_t n);        /* p8c:928-942 */
/* y[b*rows+r] = dot(row r, x[b]) + bias[r]; rows split over `threads` pthreads
 * (threads<=1: the reference's single-threaded form).  p8c:971-999 */
void orc_matmul_q4(const uint8_t *w, uint32_t n, uint32_t rows, uint32_t batch,
                   const float *x, const float *bias, float *y, int threads);
void orc_matmul_q6(const uint8_t *w, uint32_t n, uint32_t rows, uint32_t batch,
                   const float *x, const float *bias, float *y, int threads);

/* ---- elementwise / normalisation / attention ---------------------------- */
void orc_rmsnorm(const float *x, const float *w, uint32_t batch, uint32_t n,
                 float eps, float *y);                                          /* p8c:958-969 */
void orc_rope(float *x, uint32_t batch, uint32_t heads, uint32_t dim,
              uint32_t pos_base, float theta);                                  /* p8c:1001-1018 */
void orc_swiglu(const float *g, const float *u, uint32_t n, float *y);         /* p8c:1064-1073 */
void orc_add(const float *a, const float *b, uint32_t n, float *y);            /* p8c:1057-1062 */
/* cached GQA attention for one decode position over a [layer][ctx][kv_heads*dim]
 * fp32 cache.  p8c:1136-1158 */
void orc_attention_cache(const float *q, const float *kc, const float *vc,
                         uint32_t layer, uint32_t pos, uint32_t max_ctx,
                         uint32_t q_heads, uint32_t kv_heads, uint32_t dim, float *out);
/* greedy select: first index of the maximum, strict '>' (p8c:1163 argmax_ptr, and
 * src/arcllm_v1_runtime.cpp:132-148 runtime_top2 top1) */
uint32_t orc_argmax(const float *p, uint32_t n, int *finite);

/* ---- synthetic fixture streams (shared bit-for-bit with the CUDA fillers) -- */
/* n-th output of the splitmix64 sequence seeded with `seed`
 * (src/sa1_component_benchmark.cpp:71-76 is the sequential form). */
uint64_t orc_splitmix64_at(uint64_t seed, uint64_t n);
/* Q4_K super-blocks: d ~ U[1e-3,4e-3) and dmin ~ U[0,2e-3) as fp16, eight
 * 6-bit scales and mins ~ U{0..63}, 256 nibbles ~ U{0..15}. */
void orc_fill_q4k(uint8_t *dst, uint64_t block_begin, uint64_t n_blocks, uint64_t seed);
/* Q6_K super-blocks: ql/qh bytes uniform (codes ~ U{0..63}), sixteen int8
 * scales ~ U{-32..31}, d ~ U[1e-3,4e-3) as fp16. */
void orc_fill_q6k(uint8_t *dst, uint64_t block_begin, uint64_t n_blocks, uint64_t seed);
/* approximately-normal fp32 / fp16 values (Irwin-Hall sum of four 16-bit
 * uniforms, scaled to unit variance), mean mu, std sigma. */
void orc_fill_normal_f32(float *dst, uint64_t begin, uint64_t n, uint64_t seed, float mu, float sigma);
void orc_fill_normal_f16(uint16_t *dst, uint64_t begin, uint64_t n, uint64_t seed, float mu, float sigma);
/* uniform token ids in [0, vocab) */
void orc_fill_tokens(uint32_t *dst, uint64_t n, uint64_t seed, uint32_t vocab);

#ifdef __cplusplus
}
#endif
#endif
