// Internal interface of the decode-step kernels (decode_ops.cu).
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace arc {

// Device-resident greedy-decode state; the whole step reads and advances it on
// the GPU, so a captured CUDA graph replays unchanged token after token.
struct alignas(16) GreedyState {
    uint32_t token;        // token fed to the next step
    uint32_t pos;          // its position
    uint32_t n_prompt;     // prompt length
    uint32_t n_generated;  // tokens produced by greedy selection so far
    uint32_t nonfinite;    // bit 0: a non-finite logit was seen; bit 1: no finite logit
    uint32_t pad;
    unsigned long long argmax_key;  // packed (ordered value, ~index), reset by the finalize step
};

// The tensor-parallel greedy select exchanges words 4..7 (nonfinite, pad, argmax_key).
static_assert(offsetof(GreedyState, nonfinite) == 16 && offsetof(GreedyState, argmax_key) == 24,
              "GreedyState layout");

struct RopeKvShape {
    uint32_t q_heads, kv_heads, head_dim, max_ctx, layer;
};

struct AttnShape {
    uint32_t q_heads, kv_heads, head_dim, max_ctx, layer, n_splits;
    float scale;
};

// Load every decode-op kernel on the current device (before graph capture).
int decode_ops_prepare();
// ARC_OK, or the CUDA error of a launch recorded under `what`
int launch_checked(cudaError_t e, const char* what);
int launch_embed(int type, const void* table, const uint32_t* token_src, uint32_t h, uint32_t vocab, float* out,
                 cudaStream_t stream);
// rows tokens token_src[0..rows) -> out[rows][h]
int launch_embed_rows(int type, const void* table, const uint32_t* token_src, uint32_t rows, uint32_t h,
                      uint32_t vocab, float* out, cudaStream_t stream);
int launch_rope_kv_store(float* q, float* k, const float* v, const float2* table, const uint32_t* pos_src,
                         uint16_t* kc, uint16_t* vc, const RopeKvShape& s, cudaStream_t stream);
// part: scratch of kv_heads * n_splits * (q_heads/kv_heads) * (head_dim + 2) floats
// kernel launches one launch_attention call makes (1: slices merged in their cluster, 2: slices + merge)
int attention_launches(uint32_t n_splits, uint32_t q_heads, uint32_t kv_heads);
int launch_attention(const float* q, const uint16_t* kc, const uint16_t* vc, const uint32_t* pos_src,
                     const AttnShape& s, float* part, float* out, cudaStream_t stream);
// key: max over i of (ordered(logits[i]) << 32 | ~i) via atomicMax (caller zeroes it);
// nonfinite: bit 0 set when a non-finite logit is seen.
int launch_argmax(const float* logits, uint32_t n, unsigned long long* key, uint32_t* nonfinite,
                  cudaStream_t stream, uint32_t base = 0);
// Tensor-parallel greedy select: combine the ranks' gathered (nonfinite, pad, key lo, key hi)
// records (GreedyState words 4..7 of every rank) into st
int launch_greedy_combine(GreedyState* st, const uint32_t* recs, uint32_t n_ranks, cudaStream_t stream);
int launch_greedy_finalize(GreedyState* st, const uint32_t* prompt, uint32_t* out_tokens, uint32_t max_out,
                           cudaStream_t stream);

}  // namespace arc
