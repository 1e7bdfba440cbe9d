// Internal interface of the batched prefill kernels (prefill_ops.cu).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "decode_ops.h"

namespace arc {

// out[r][i] = v rounded to bf16 (or fp16 when `fp16`; an overflow sets the
// device error word's range bit), v = (x[r][i] * rsqrt(mean_i(x[r]^2) + eps)) * gamma[i];
// fp16 only: out_lo (nullable) = fp16(v - out)
int launch_rmsnorm_rows_bf16(const float* x, const float* gamma, float eps, uint32_t rows, uint32_t h, uint16_t* out,
                             cudaStream_t stream, bool fp16 = false, uint16_t* out_lo = nullptr);
// rows t of q[rows][q_heads*hd], k, v[rows][kv_dim] (+ biases, nullable): RoPE
// at position pos0+t, q and k rotated in place, k and v stored to the fp16 cache
int launch_rope_kv_rows(float* q, float* k, const float* v, const float* bq, const float* bk, const float* bv,
                        const float2* table, uint32_t pos0, uint32_t rows, uint16_t* kc, uint16_t* vc,
                        const RopeKvShape& s, cudaStream_t stream);
// causal attention of query rows t over cache positions 0..pos0+t -> out bf16 [rows][q_heads*hd]
int launch_attention_prefill(const float* q, const uint16_t* kc, const uint16_t* vc, uint32_t pos0, uint32_t rows,
                             const AttnShape& s, uint16_t* out, cudaStream_t stream);
// decode state after a batched prefill of positions 0 .. n_prompt-2
int launch_prefill_done(GreedyState* st, const uint32_t* prompt, uint32_t n_prompt, cudaStream_t stream);
// out[i] = bf16(silu(g[i]) * u[i])
int launch_silu_mul_rows_bf16(const float* g, const float* u, uint64_t n, uint16_t* out, cudaStream_t stream);

}  // namespace arc
