/*
 * C-ABI exports of the reference's OWN CPU functions, compiled in place from
 * the ArcLLM sources (nothing is copied: the reference files are #included
 * from the path given with -I by oracle/build.py, and the output goes to
 * oracle/_ref/).  TEST INFRASTRUCTURE ONLY: used to generate
 * tests/golden/ and to pin the C restatement in oracle/orc.c.
 *
 *   src/p8c_segmented_access_correctness.cpp  -- half_to_float (503),
 *       scale_min_cpu (531), q4k_dot_row (542), q6_value_cpu (905),
 *       q6k_dot_row (928), q6k_dequant_row (944), rmsnorm_cpu (958),
 *       matmul_q4_cpu (971), matmul_q6_cpu (986), rope_cpu (1001),
 *       add_cpu (1057), swiglu_cpu (1064), attention_cache_cpu (1136),
 *       argmax_ptr (1163), q4k_dequant_row_p8c (1166)
 *   src/q6cb_q6_reference.hpp                 -- decode_q6_element (49-91)
 *   src/q6cb_fixture_generator.hpp            -- generate_fixture (160-193),
 *       verify_semantic_invariant (196-229)
 *   src/q4_down_exec148_materializer.h        -- materialize_block,
 *       validator tuples, Sha256 (12-22)
 */
#include <cstdint>
#include <cstring>
#include <vector>

#define main static arcllm_p8c_reference_main_unused
#include "p8c_segmented_access_correctness.cpp"
#undef main
#include "q6cb_fixture_generator.hpp"
#include "q4_down_exec148_materializer.h"

extern "C" {

float ref_half_to_float(uint16_t h) { return half_to_float(h); }

void ref_q4k_scale_min(const uint8_t* b, int j, uint8_t* sc, uint8_t* mn) {
    scale_min_cpu(b, j, *sc, *mn);
}

void ref_q4k_dequant_row(const uint8_t* row, float* y, uint32_t n) { q4k_dequant_row_p8c(row, y, n); }
void ref_q6k_dequant_row(const uint8_t* row, float* y, uint32_t n) { q6k_dequant_row(row, y, n); }
float ref_q4k_dot_row(const uint8_t* row, const float* x, uint32_t n) { return q4k_dot_row(row, x, n); }
float ref_q6k_dot_row(const uint8_t* row, const float* x, uint32_t n) { return q6k_dot_row(row, x, n); }

void ref_matmul_q4(const uint8_t* w, uint32_t n, uint32_t rows, uint32_t batch,
                   const float* x, const float* bias, float* y) {
    std::vector<float> xv(x, x + size_t(batch) * n);
    std::vector<float> out = matmul_q4_cpu(w, n, rows, batch, xv, bias);
    std::memcpy(y, out.data(), out.size() * sizeof(float));
}

void ref_matmul_q6(const uint8_t* w, uint32_t n, uint32_t rows, uint32_t batch,
                   const float* x, const float* bias, float* y) {
    std::vector<float> xv(x, x + size_t(batch) * n);
    std::vector<float> out = matmul_q6_cpu(w, n, rows, batch, xv, bias);
    std::memcpy(y, out.data(), out.size() * sizeof(float));
}

void ref_rmsnorm(const float* x, const float* w, uint32_t batch, uint32_t n, float eps, float* y) {
    std::vector<float> xv(x, x + size_t(batch) * n);
    std::vector<float> out = rmsnorm_cpu(xv, w, batch, n, eps);
    std::memcpy(y, out.data(), out.size() * sizeof(float));
}

void ref_rope(float* x, uint32_t batch, uint32_t heads, uint32_t dim, uint32_t pos_base, float theta) {
    std::vector<float> xv(x, x + size_t(batch) * heads * dim);
    rope_cpu(xv, batch, heads, dim, pos_base, theta);
    std::memcpy(x, xv.data(), xv.size() * sizeof(float));
}

void ref_swiglu(const float* g, const float* u, uint32_t n, float* y) {
    std::vector<float> gv(g, g + n), uv(u, u + n);
    std::vector<float> out = swiglu_cpu(gv, uv);
    std::memcpy(y, out.data(), n * sizeof(float));
}

void ref_add(const float* a, const float* b, uint32_t n, float* y) {
    std::vector<float> av(a, a + n), bv(b, b + n);
    std::vector<float> out = add_cpu(av, bv);
    std::memcpy(y, out.data(), n * sizeof(float));
}

void ref_attention_cache(const float* q, const float* kc, const float* vc, uint64_t cache_elems,
                         uint32_t layer, uint32_t pos, uint32_t max_ctx, uint32_t q_heads,
                         uint32_t kv_heads, uint32_t dim, float* out) {
    std::vector<float> qv(q, q + size_t(q_heads) * dim);
    std::vector<float> kv(kc, kc + cache_elems), vv(vc, vc + cache_elems);
    std::vector<float> o = attention_cache_cpu(qv, kv, vv, layer, pos, max_ctx, q_heads, kv_heads, dim);
    std::memcpy(out, o.data(), o.size() * sizeof(float));
}

uint32_t ref_argmax(const float* p, uint32_t n, int* finite) {
    bool f = false;
    uint32_t i = argmax_ptr(p, n, f);
    if (finite) *finite = f ? 1 : 0;
    return i;
}

/* src/q6cb_q6_reference.hpp:49-91 -- canonical Q6_K element decode */
float ref_q6cb_decode_value(const uint8_t* block, uint32_t k, int* q, int* scale) {
    q6cb::CanonicalQ6Element e = q6cb::decode_q6_element(block, k);
    if (q) *q = e.q;
    if (scale) *scale = e.scale;
    return e.value;
}

/* src/q6cb_fixture_generator.hpp:160-229 -- deterministic Q6_K packer over the
 * conditioning strata, plus its semantic invariant.  Returns 1 if the
 * invariant passes.  `packed` must hold rows*(n/256)*210 bytes, `x` n floats. */
int ref_q6cb_fixture(uint32_t n, uint32_t rows, uint64_t seed, int stratum,
                     uint8_t* packed, float* x) {
    q6cb::FixtureSpec s;
    s.id = "arcllm-b200-golden";
    s.n = n;
    s.rows = rows;
    s.seed = seed;
    s.stratum = static_cast<q6cb::ConditioningStratum>(stratum);
    q6cb::Fixture f = q6cb::generate_fixture(s);
    std::memcpy(packed, f.packed.data(), f.packed.size());
    std::memcpy(x, f.x.data(), f.x.size() * sizeof(float));
    return q6cb::verify_semantic_invariant(f).pass ? 1 : 0;
}

/* src/q4_down_exec148_materializer.h -- Q4_K (144 B) -> EXEC148 (148 B) */
void ref_exec148_materialize_block(const uint8_t* src, uint8_t* dst) {
    arcllm_exec148::materialize_block(src, dst);
}

void ref_exec148_source_tuple(const uint8_t* src, uint8_t* out276) {
    std::array<uint8_t, arcllm_exec148::kCanonicalBytes> t{};
    arcllm_exec148::validator_source_tuple(src, t);
    std::memcpy(out276, t.data(), t.size());
}

void ref_sha256(const uint8_t* p, uint64_t n, uint8_t* out32) {
    arcllm_exec148::Sha256 h;
    h.update(p, size_t(n));
    std::array<uint8_t, 32> d = h.final();
    std::memcpy(out32, d.data(), 32);
}

}  // extern "C"
