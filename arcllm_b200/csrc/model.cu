// Greedy decode runtime for one Qwen2-family model on one GPU, behind the C ABI.
//
// This is the device half of the reference's generate()
// (src/arcllm_v1_runtime.cpp:149-536): its per-token Vulkan chain of 469
// dispatches with a fence wait and a host top-2 per token (:371-421, 461-505)
// becomes one CUDA-graph launch per token whose kernels read the position and
// token from device memory and write the next token back on the device
// (greedy argmax included), so consecutive tokens need no host round trip.
//
// Per layer (decode_step): RMSNorm fused into the Q/K/V matvecs (+bias),
// RoPE + fp16 KV store, split-KV GQA attention, O projection + residual,
// RMSNorm fused into the dual gate/up matvec with silu(g)*u, down projection
// + residual.  Then output RMSNorm fused into the LM head, argmax, finalize.
// The prompt (all but its last token) is consumed in batches of up to 256
// rows on the tensor cores (enqueue_prefill_chunk: tcgen05 GEMMs for every
// projection, fp16 hi + lo operands for Q/K/V and bf16 for the rest, batched RMSNorm / RoPE + KV store / causal attention /
// SiLU kernels -- the reference's prefill chain, src/arcllm_v1_runtime.cpp:
// 340-369), or, in prefill mode 0, token by token through the decode layer
// chain without the LM head (the prefill graph, fp32 throughout).
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <new>
#include <vector>

#include "arcllm_cuda_internal.h"
#include "decode_ops.h"
#include "prefill_ops.h"

struct arcllm_cuda_model {
    int device = 0;
    arcllm_cuda_model_config cfg{};
    std::vector<arcllm_cuda_layer> layers;
    std::vector<uint8_t> layer_set;
    const void* tok_embd = nullptr;
    int tok_embd_type = 0;
    const float* out_norm = nullptr;
    const void* out_w = nullptr;
    int out_type = 0;
    bool endpoints_set = false;
    // row shard of the LM head computed here (all rows unless sharded)
    uint32_t lm_row0 = 0, lm_rows = 0;

    // device memory (one allocation)
    void* arena = nullptr;
    float *h0 = nullptr, *h1 = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *attn = nullptr, *s = nullptr,
          *logits = nullptr, *part = nullptr;
    uint16_t *kc = nullptr, *vc = nullptr;
    float2* rope = nullptr;
    arc::GreedyState* state = nullptr;
    uint32_t* prompt = nullptr;
    uint32_t* out_tokens = nullptr;
    uint32_t attn_splits = 16;

    cudaGraphExec_t g_prefill = nullptr, g_decode = nullptr;
    uint32_t launches_prefill_step = 0, launches_decode_step = 0;
    // K and V projections run beside Q on two side streams (forked and joined with events)
    cudaStream_t side[2] = {nullptr, nullptr};
    cudaEvent_t ev_fork = nullptr, ev_join[2] = {nullptr, nullptr};

    // batched prefill (allocated on first use): rows of up to kPrefillRows prompt tokens
    int prefill_mode = 1;  // 1: tensor-core batches; 0: token by token
    std::vector<const void*> prefill_down;  // Q4_K/Q6_K down weights when w_down is an EXEC148 image
    std::vector<int> prefill_down_type;
    void* pf_arena = nullptr;
    float *pf_h = nullptr, *pf_h2 = nullptr, *pf_q = nullptr, *pf_k = nullptr, *pf_v = nullptr, *pf_g = nullptr,
          *pf_u = nullptr;
    uint16_t *pf_xb = nullptr, *pf_xb_lo = nullptr, *pf_attn = nullptr, *pf_s = nullptr;
    uint32_t launches_prefill_batched = 0;
    uint32_t begun_prompt = 0;  // prompt length of the last begin() (0: none)

    // tensor parallelism (tp.n_ranks > 1): this rank's FFN gate/up rows [ffn_r0, +ffn_rows) --
    // the same range of s is its K window of the FFN down projection -- (its LM-head rows are
    // lm_row0/lm_rows), the ranks' exchange buffers, the down projection's partial sums and
    // the gathered greedy records (4 words per rank)
    arc::ExchangeRanks tp{};
    uint32_t ffn_r0 = 0, ffn_rows = 0;
    float* tp_part = nullptr;
    uint32_t* tp_recs = nullptr;
};

namespace arc {
namespace {

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

bool quant_ok(int t) { return t == ARC_GGML_Q4_K || t == ARC_GGML_Q6_K; }

// Bytes of one row of k weights (Q4_K, Q6_K or the EXEC148 image).
uint64_t row_bytes(int type, uint32_t k) {
    const uint64_t blk = type == ARC_GGML_Q4_K ? 144u : type == ARC_GGML_Q6_K ? 210u : 148u;
    return (uint64_t)(k / 256u) * blk;
}

// Rows of a tensor-parallel shard are whole 32-row groups (the matvecs' row
// groups; keeps every shard's weight rows and vector slices 16-byte aligned).
constexpr uint32_t kTpRowAlign = 32;
constexpr uint32_t kTpFfnAlign = 512;  // FFN shards: pairs of 256-weight super-blocks

int check_layer(const arcllm_cuda_model_config& c, const arcllm_cuda_layer& L) {
    if (!L.attn_norm || !L.ffn_norm || !L.wq || !L.wk || !L.wv || !L.wo || !L.w_gate || !L.w_up || !L.w_down)
        return set_error(ARC_E_INVALID_ARGUMENT, "model_set_layer: null tensor pointer");
    if (!quant_ok(L.type_q) || !quant_ok(L.type_k) || !quant_ok(L.type_v) || !quant_ok(L.type_o) ||
        !(quant_ok(L.type_down) || L.type_down == ARC_TYPE_EXEC148) || L.type_gate_up != ARC_GGML_Q4_K)
        return set_error(ARC_E_UNSUPPORTED_SHAPE,
                         "model_set_layer: projections must be Q4_K/Q6_K and gate/up Q4_K "
                         "(reference contract: src/arcllm_v1_runtime.cpp:194-211)");
    (void)c;
    return ARC_OK;
}

// Launch one matvec with a freshly computed plan (host-only arithmetic).
int mv(int type, const void* w, uint32_t rows, uint32_t k, const float* x, const float* gamma, float eps,
       const float* bias, const float* residual, float* y, cudaStream_t st) {
    return matvec_any(type, false, w, nullptr, rows, k, x, gamma, eps, bias, residual, y, st);
}

#define ARC_TRY(expr)          \
    do {                       \
        int _st = (expr);      \
        if (_st != ARC_OK) return _st; \
    } while (0)

// RoPE + KV store can ride in the Q/K/V matvec epilogues: all three on the
// whole-row integer-MMA kernel (K <= 3584, 16-byte aligned x and gamma).
bool fuse_rope_ok(const arcllm_cuda_model* m, const arcllm_cuda_layer& L) {
    if (const char* e = std::getenv("ARCLLM_FUSE_ROPE"))
        if (std::strcmp(e, "0") == 0) return false;
    if (std::getenv("ARCLLM_MATVEC_IMPL") && std::strcmp(std::getenv("ARCLLM_MATVEC_IMPL"), "cuda") == 0) return false;
    const arcllm_cuda_model_config& c = m->cfg;
    const uint32_t H = c.hidden, KV = c.n_kv_heads * c.head_dim;
    if ((reinterpret_cast<uintptr_t>(L.attn_norm) & 15u) != 0u) return false;
    return matvec_imma_supported(L.type_q, false, H, H) && matvec_imma_supported(L.type_k, false, KV, H) &&
           matvec_imma_supported(L.type_v, false, KV, H);
}

// Q, K and V as one launch (matvec_imma_multi_launch) where it applies; ARCLLM_QKV_ONE_LAUNCH=0
// keeps three launches, K and V on side streams.
bool qkv_one_launch() {
    static const bool on = [] {
        const char* e = std::getenv("ARCLLM_QKV_ONE_LAUNCH");
        return !(e && e[0] == '0');
    }();
    return on;
}

// Enqueue one token step; `with_head` adds output norm + LM head + argmax.
int enqueue_step(arcllm_cuda_model* m, bool with_head, cudaStream_t st, uint32_t* n_launch) {
    const arcllm_cuda_model_config& c = m->cfg;
    const uint32_t H = c.hidden, KV = c.n_kv_heads * c.head_dim;
    uint32_t n = 0;
    ARC_TRY(launch_embed(m->tok_embd_type, m->tok_embd, &m->state->token, H, c.vocab, m->h0, st));
    ++n;
    float* hc = m->h0;
    float* hm = m->h1;
    for (uint32_t l = 0; l < c.n_layers; ++l) {
        const arcllm_cuda_layer& L = m->layers[l];
        // RoPE and the fp16 KV store ride in the Q/K/V matvec epilogues when the whole-row
        // integer-MMA kernel takes all three (ARCLLM_FUSE_ROPE=0 keeps the separate kernel)
        const bool fuse = fuse_rope_ok(m, L);
        const uint64_t lcache = (uint64_t)l * c.max_ctx * KV;
        const uint32_t half = c.head_dim / 2u;
        const RopeEpilogue rq{1u, half, c.max_ctx, m->rope, &m->state->pos, nullptr};
        const RopeEpilogue rk{2u, half, c.max_ctx, m->rope, &m->state->pos, m->kc + lcache};
        const RopeEpilogue rv{3u, half, c.max_ctx, m->rope, &m->state->pos, m->vc + lcache};
        const ImmaJob qkv[3] = {{L.type_q, L.wq, H, L.bq, m->q, &rq},
                                {L.type_k, L.wk, KV, L.bk, m->k, &rk},
                                {L.type_v, L.wv, KV, L.bv, m->v, &rv}};
        if (fuse && qkv_one_launch() && matvec_imma_multi_supported(qkv, H)) {
            // Q, K and V read the same input: one grid (112 + 16 + 16 CTAs at the Qwen2.5-7B
            // shape), so the attention follows it with programmatic dependent launch
            ARC_TRY(matvec_imma_multi_launch(qkv, H, hc, L.attn_norm, c.rms_eps, st));
            n += 1;
        } else {
            // otherwise K and V go to side streams so the three matvecs share the GPU
            ARC_TRY(launch_checked(cudaEventRecord(m->ev_fork, st), "fork"));
            for (int i = 0; i < 2; ++i)
                ARC_TRY(launch_checked(cudaStreamWaitEvent(m->side[i], m->ev_fork, 0), "fork"));
            if (fuse)
                ARC_TRY(matvec_imma_launch(L.type_q, false, L.wq, nullptr, H, H, hc, L.attn_norm, c.rms_eps, L.bq,
                                           nullptr, m->q, st, &rq));
            else
                ARC_TRY(mv(L.type_q, L.wq, H, H, hc, L.attn_norm, c.rms_eps, L.bq, nullptr, m->q, st));
            {
                PdlScope plain(false);  // a side stream's predecessor is an event, not a kernel
                if (fuse) {
                    ARC_TRY(matvec_imma_launch(L.type_k, false, L.wk, nullptr, KV, H, hc, L.attn_norm, c.rms_eps,
                                               L.bk, nullptr, m->k, m->side[0], &rk));
                    ARC_TRY(matvec_imma_launch(L.type_v, false, L.wv, nullptr, KV, H, hc, L.attn_norm, c.rms_eps,
                                               L.bv, nullptr, m->v, m->side[1], &rv));
                } else {
                    ARC_TRY(mv(L.type_k, L.wk, KV, H, hc, L.attn_norm, c.rms_eps, L.bk, nullptr, m->k,
                               m->side[0]));
                    ARC_TRY(mv(L.type_v, L.wv, KV, H, hc, L.attn_norm, c.rms_eps, L.bv, nullptr, m->v,
                               m->side[1]));
                }
            }
            for (int i = 0; i < 2; ++i) {
                ARC_TRY(launch_checked(cudaEventRecord(m->ev_join[i], m->side[i]), "join"));
                ARC_TRY(launch_checked(cudaStreamWaitEvent(st, m->ev_join[i], 0), "join"));
            }
            if (!fuse) {
                RopeKvShape rs{c.n_heads, c.n_kv_heads, c.head_dim, c.max_ctx, l};
                ARC_TRY(launch_rope_kv_store(m->q, m->k, m->v, m->rope, &m->state->pos, m->kc, m->vc, rs, st));
                ++n;
            }
            n += 3;
        }
        AttnShape as{c.n_heads, c.n_kv_heads, c.head_dim, c.max_ctx, l, m->attn_splits,
                     1.0f / std::sqrt((float)c.head_dim)};
        ARC_TRY(launch_attention(m->q, m->kc, m->vc, &m->state->pos, as, m->part, m->attn, st));
        ARC_TRY(mv(L.type_o, L.wo, H, H, m->attn, nullptr, 0.f, nullptr, hc, hm, st));
        n += 1 + (uint32_t)attention_launches(m->attn_splits, c.n_heads, c.n_kv_heads);  // (attn) O
        if (m->tp.n_ranks > 1) {
            // this rank's gate/up rows -> its slice of s; the FFN down over the same K window
            // (every output row, this slice's super-blocks) -> partial sums; the ranks' partials
            // added in rank order plus the residual on every rank (one exchange per layer)
            const uint64_t rb_gu = row_bytes(ARC_GGML_Q4_K, H);
            const uint8_t* wg = static_cast<const uint8_t*>(L.w_gate) + (uint64_t)m->ffn_r0 * rb_gu;
            const uint8_t* wu = static_cast<const uint8_t*>(L.w_up) + (uint64_t)m->ffn_r0 * rb_gu;
            ARC_TRY(matvec_any(ARC_GGML_Q4_K, true, wg, wu, m->ffn_rows, H, hm, L.ffn_norm, c.rms_eps, nullptr,
                               nullptr, m->s + m->ffn_r0, st));
            ARC_TRY(matvec_kwindow_launch(L.type_down, L.w_down, H, c.ffn, m->ffn_r0 / 256u, m->ffn_rows / 256u,
                                          m->s, nullptr, 0.f, nullptr, nullptr, m->tp_part, st));
            ARC_TRY(exchange_reduce(m->tp, m->tp_part, H, hm, hc, st));
            n += 3;
        } else {
            ARC_TRY(matvec_any(ARC_GGML_Q4_K, true, L.w_gate, L.w_up, c.ffn, H, hm, L.ffn_norm, c.rms_eps, nullptr,
                               nullptr, m->s, st));
            ARC_TRY(mv(L.type_down, L.w_down, H, c.ffn, m->s, nullptr, 0.f, nullptr, hm, hc, st));
            n += 2;
        }
    }
    if (with_head) {
        const uint8_t* wo = static_cast<const uint8_t*>(m->out_w) + (uint64_t)m->lm_row0 * row_bytes(m->out_type, H);
        ARC_TRY(mv(m->out_type, wo, m->lm_rows, H, hc, m->out_norm, c.rms_eps, nullptr, nullptr,
                   m->logits + m->lm_row0, st));
        n += 2;
        if (m->tp.n_ranks > 1) {
            // the shard's argmax over global row indices, then the ranks' records gathered and combined
            ARC_TRY(launch_argmax(m->logits + m->lm_row0, m->lm_rows, &m->state->argmax_key, &m->state->nonfinite,
                                  st, m->lm_row0));
            ARC_TRY(exchange_gather(m->tp, reinterpret_cast<const uint32_t*>(m->state) + 4, 4u, 4u * m->tp.rank,
                                    m->tp_recs, 4u * m->tp.n_ranks, st));
            ARC_TRY(launch_greedy_combine(m->state, m->tp_recs, m->tp.n_ranks, st));
            n += 2;
        } else {
            ARC_TRY(launch_argmax(m->logits, c.vocab, &m->state->argmax_key, &m->state->nonfinite, st));
        }
    }
    ARC_TRY(launch_greedy_finalize(m->state, m->prompt, m->out_tokens, c.max_ctx, st));
    ++n;
    if (n_launch) *n_launch = n;
    return ARC_OK;
}

int capture(arcllm_cuda_model* m, bool with_head, cudaGraphExec_t* out, uint32_t* n_launch) {
    cudaStream_t cs;
    cudaError_t e = cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking);
    if (e != cudaSuccess) return set_cuda_error(e, "capture stream");
    e = cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) {
        cudaStreamDestroy(cs);
        return set_cuda_error(e, "begin capture");
    }
    int st;
    {
        PdlScope pdl(true);  // weights are constant for the graph's lifetime
        st = enqueue_step(m, with_head, cs, n_launch);
    }
    cudaGraph_t g = nullptr;
    e = cudaStreamEndCapture(cs, &g);
    cudaStreamDestroy(cs);
    if (st != ARC_OK) {
        if (g) cudaGraphDestroy(g);
        return st;
    }
    if (e != cudaSuccess) return set_cuda_error(e, "end capture");
    e = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return set_cuda_error(e, "graph instantiate");
    return ARC_OK;
}

constexpr uint32_t kPrefillRows = 256;  // the GEMMs' M limit

// Down weights of layer l for the batched prefill (the GEMM reads Q4_K/Q6_K,
// not the EXEC148 image); null when none is available.
const void* prefill_down_w(const arcllm_cuda_model* m, uint32_t l, int* type) {
    const arcllm_cuda_layer& L = m->layers[l];
    if (L.type_down != ARC_TYPE_EXEC148) {
        *type = L.type_down;
        return L.w_down;
    }
    *type = m->prefill_down_type[l];
    return m->prefill_down[l];
}

bool prefill_batched_ok(const arcllm_cuda_model* m) {
    if (m->prefill_mode != 1) return false;
    if (const char* e = std::getenv("ARCLLM_PREFILL"))
        if (std::strcmp(e, "token") == 0) return false;
    for (uint32_t l = 0; l < m->cfg.n_layers; ++l) {
        int t = 0;
        if (!prefill_down_w(m, l, &t) || !quant_ok(t)) return false;
    }
    return true;
}

int prefill_alloc(arcllm_cuda_model* m) {
    if (m->pf_arena) return ARC_OK;
    const arcllm_cuda_model_config& c = m->cfg;
    const size_t T = kPrefillRows, H = c.hidden, KV = (size_t)c.n_kv_heads * c.head_dim, F = c.ffn;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off = align_up(off + bytes, 256);
        return o;
    };
    const size_t o_h = take(4 * T * H), o_h2 = take(4 * T * H), o_q = take(4 * T * H), o_k = take(4 * T * KV),
                 o_v = take(4 * T * KV), o_g = take(4 * T * F), o_u = take(4 * T * F), o_xb = take(2 * T * H),
                 o_xb_lo = take(2 * T * H), o_attn = take(2 * T * H), o_s = take(2 * T * F);
    const cudaError_t e = cudaMalloc(&m->pf_arena, off);
    if (e != cudaSuccess) {
        m->pf_arena = nullptr;
        return set_cuda_error(e, "prefill buffers");
    }
    uint8_t* a = static_cast<uint8_t*>(m->pf_arena);
    m->pf_h = reinterpret_cast<float*>(a + o_h);
    m->pf_h2 = reinterpret_cast<float*>(a + o_h2);
    m->pf_q = reinterpret_cast<float*>(a + o_q);
    m->pf_k = reinterpret_cast<float*>(a + o_k);
    m->pf_v = reinterpret_cast<float*>(a + o_v);
    m->pf_g = reinterpret_cast<float*>(a + o_g);
    m->pf_u = reinterpret_cast<float*>(a + o_u);
    m->pf_xb = reinterpret_cast<uint16_t*>(a + o_xb);
    m->pf_xb_lo = reinterpret_cast<uint16_t*>(a + o_xb_lo);
    m->pf_attn = reinterpret_cast<uint16_t*>(a + o_attn);
    m->pf_s = reinterpret_cast<uint16_t*>(a + o_s);
    return ARC_OK;
}

// Prompt rows pos0 .. pos0+T-1 through every layer: their K/V land in the
// cache; the hidden states themselves are not kept (no LM head for them).
int enqueue_prefill_chunk(arcllm_cuda_model* m, uint32_t pos0, uint32_t T, cudaStream_t st, uint32_t* n_launch) {
    const arcllm_cuda_model_config& c = m->cfg;
    const uint32_t H = c.hidden, KV = c.n_kv_heads * c.head_dim, F = c.ffn;
    uint32_t n = 0;
    ARC_TRY(launch_embed_rows(m->tok_embd_type, m->tok_embd, m->prompt + pos0, T, H, c.vocab, m->pf_h, st));
    ++n;
    for (uint32_t l = 0; l < c.n_layers; ++l) {
        const arcllm_cuda_layer& L = m->layers[l];
        int type_down = 0;
        const void* w_down = prefill_down_w(m, l, &type_down);
        // Q, K and V feed the attention scores, which the synthetic models make nearly one-hot
        // (q.k/sqrt(d) of 1e3-1e4): their GEMMs take fp16 hi + lo halves of both operands
        // (~22 bits; bf16's or a single fp16's rounding of the weights moved near-tied
        // positions of long prompts), the other GEMMs bf16
        ARC_TRY(launch_rmsnorm_rows_bf16(m->pf_h, L.attn_norm, c.rms_eps, T, H, m->pf_xb, st, true, m->pf_xb_lo));
        ARC_TRY(gemm_kq_bf16(L.type_q, L.wq, H, H, m->pf_xb, T, nullptr, m->pf_q, st, 2, m->pf_xb_lo));
        ARC_TRY(gemm_kq_bf16(L.type_k, L.wk, KV, H, m->pf_xb, T, nullptr, m->pf_k, st, 2, m->pf_xb_lo));
        ARC_TRY(gemm_kq_bf16(L.type_v, L.wv, KV, H, m->pf_xb, T, nullptr, m->pf_v, st, 2, m->pf_xb_lo));
        RopeKvShape rs{c.n_heads, c.n_kv_heads, c.head_dim, c.max_ctx, l};
        ARC_TRY(launch_rope_kv_rows(m->pf_q, m->pf_k, m->pf_v, L.bq, L.bk, L.bv, m->rope, pos0, T, m->kc, m->vc, rs,
                                    st));
        AttnShape as{c.n_heads, c.n_kv_heads, c.head_dim, c.max_ctx, l, 1, 1.0f / std::sqrt((float)c.head_dim)};
        ARC_TRY(launch_attention_prefill(m->pf_q, m->kc, m->vc, pos0, T, as, m->pf_attn, st));
        ARC_TRY(gemm_kq_bf16(L.type_o, L.wo, H, H, m->pf_attn, T, m->pf_h, m->pf_h2, st));  // h2 = h + O
        ARC_TRY(launch_rmsnorm_rows_bf16(m->pf_h2, L.ffn_norm, c.rms_eps, T, H, m->pf_xb, st));
        ARC_TRY(gemm_kq_bf16(ARC_GGML_Q4_K, L.w_gate, F, H, m->pf_xb, T, nullptr, m->pf_g, st));
        ARC_TRY(gemm_kq_bf16(ARC_GGML_Q4_K, L.w_up, F, H, m->pf_xb, T, nullptr, m->pf_u, st));
        ARC_TRY(launch_silu_mul_rows_bf16(m->pf_g, m->pf_u, (uint64_t)T * F, m->pf_s, st));
        ARC_TRY(gemm_kq_bf16(type_down, w_down, H, F, m->pf_s, T, m->pf_h2, m->pf_h, st));  // h = h2 + down
        n += 12;
    }
    if (n_launch) *n_launch += n;
    return ARC_OK;
}

}  // namespace

// RoPE table: cos/sin of pos * theta^(-2p/d) computed with the reference's
// float expression (src/p8c_segmented_access_correctness.cpp:1010-1011).
std::vector<float> rope_table(uint32_t max_ctx, uint32_t head_dim, float theta) {
    const uint32_t half = head_dim / 2u;
    std::vector<float> t((size_t)max_ctx * half * 2u);
    for (uint32_t pos = 0; pos < max_ctx; ++pos) {
        for (uint32_t p = 0; p < half; ++p) {
            volatile float ex = -2.0f * (float)p;
            ex = ex / (float)head_dim;
            volatile float pw = std::pow(theta, (float)ex);
            volatile float angle = (float)pos * (float)pw;
            t[((size_t)pos * half + p) * 2 + 0] = std::cos((float)angle);
            t[((size_t)pos * half + p) * 2 + 1] = std::sin((float)angle);
        }
    }
    return t;
}

int model_create(const arcllm_cuda_model_config* cfg, arcllm_cuda_model** out) {
    if (!cfg || !out) return set_error(ARC_E_INVALID_ARGUMENT, "model_create: null pointer");
    const arcllm_cuda_model_config& c = *cfg;
    if (c.n_layers == 0 || c.hidden == 0 || c.hidden % 256u || c.ffn % 256u || c.ffn == 0 || c.head_dim != 128u ||
        c.n_heads == 0 || c.n_kv_heads == 0 || c.n_heads % c.n_kv_heads || c.n_heads * c.head_dim != c.hidden ||
        c.vocab == 0 || c.max_ctx == 0)
        return set_error(ARC_E_UNSUPPORTED_SHAPE,
                         "model_create: needs hidden,ffn multiples of 256, head_dim 128, heads*head_dim == hidden");
    ARC_TRY(matvec_prepare());
    ARC_TRY(matvec_imma_prepare());
    ARC_TRY(matvec_splitk_prepare());
    // FFN down scratch for the K-slice kernel, before any graph capture (either format)
    ARC_TRY(matvec_splitk_reserve(ARC_GGML_Q4_K, cfg->hidden, cfg->ffn));
    ARC_TRY(matvec_splitk_reserve(ARC_GGML_Q6_K, cfg->hidden, cfg->ffn));
    ARC_TRY(matvec_splitk_reserve(ARC_TYPE_EXEC148, cfg->hidden, cfg->ffn));
    ARC_TRY(decode_ops_prepare());
    if (!dev_error_word()) return set_error(ARC_E_CUDA, "model_create: device error word unavailable");
    auto* m = new (std::nothrow) arcllm_cuda_model();
    if (!m) return set_error(ARC_E_OUT_OF_MEMORY, "model_create: host allocation");
    cudaGetDevice(&m->device);
    m->cfg = c;
    m->layers.resize(c.n_layers);
    m->layer_set.assign(c.n_layers, 0);
    m->prefill_down.assign(c.n_layers, nullptr);
    m->prefill_down_type.assign(c.n_layers, 0);
    m->lm_row0 = 0;
    m->lm_rows = c.vocab;
    // tuning override for experiments: ARCLLM_ATTN_SPLITS=<KV slices per head> (1 .. 64)
    if (const char* e = std::getenv("ARCLLM_ATTN_SPLITS")) {
        const unsigned long v = std::strtoul(e, nullptr, 10);
        if (v >= 1 && v <= 64) m->attn_splits = (uint32_t)v;
    }
    const uint32_t gq = c.n_heads / c.n_kv_heads;
    const size_t kv_dim = (size_t)c.n_kv_heads * c.head_dim;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off = align_up(off + bytes, 256);
        return o;
    };
    const size_t o_h0 = take(4 * c.hidden), o_h1 = take(4 * c.hidden), o_q = take(4 * c.hidden),
                 o_k = take(4 * kv_dim), o_v = take(4 * kv_dim), o_attn = take(4 * c.hidden),
                 o_s = take(4 * (size_t)c.ffn), o_logits = take(4 * (size_t)c.vocab),
                 o_part = take(4 * (size_t)c.n_kv_heads * m->attn_splits * gq * (c.head_dim + 2)),
                 o_kc = take(2 * (size_t)c.n_layers * c.max_ctx * kv_dim),
                 o_vc = take(2 * (size_t)c.n_layers * c.max_ctx * kv_dim),
                 o_rope = take(8 * (size_t)c.max_ctx * (c.head_dim / 2)), o_state = take(sizeof(GreedyState)),
                 o_prompt = take(4 * (size_t)c.max_ctx), o_out = take(4 * (size_t)c.max_ctx);
    cudaError_t e = cudaMalloc(&m->arena, off);
    if (e != cudaSuccess) {
        delete m;
        return set_cuda_error(e, "model_create: device arena");
    }
    uint8_t* a = static_cast<uint8_t*>(m->arena);
    m->h0 = reinterpret_cast<float*>(a + o_h0);
    m->h1 = reinterpret_cast<float*>(a + o_h1);
    m->q = reinterpret_cast<float*>(a + o_q);
    m->k = reinterpret_cast<float*>(a + o_k);
    m->v = reinterpret_cast<float*>(a + o_v);
    m->attn = reinterpret_cast<float*>(a + o_attn);
    m->s = reinterpret_cast<float*>(a + o_s);
    m->logits = reinterpret_cast<float*>(a + o_logits);
    m->part = reinterpret_cast<float*>(a + o_part);
    m->kc = reinterpret_cast<uint16_t*>(a + o_kc);
    m->vc = reinterpret_cast<uint16_t*>(a + o_vc);
    m->rope = reinterpret_cast<float2*>(a + o_rope);
    m->state = reinterpret_cast<GreedyState*>(a + o_state);
    m->prompt = reinterpret_cast<uint32_t*>(a + o_prompt);
    m->out_tokens = reinterpret_cast<uint32_t*>(a + o_out);
    std::vector<float> rt = rope_table(c.max_ctx, c.head_dim, c.rope_theta);
    e = cudaMemcpy(m->rope, rt.data(), rt.size() * sizeof(float), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(m->logits, 0, 4 * (size_t)c.vocab);
    if (e != cudaSuccess) {
        cudaFree(m->arena);
        delete m;
        return set_cuda_error(e, "model_create: init");
    }
    for (int i = 0; i < 2 && e == cudaSuccess; ++i) e = cudaStreamCreateWithFlags(&m->side[i], cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&m->ev_fork, cudaEventDisableTiming);
    for (int i = 0; i < 2 && e == cudaSuccess; ++i) e = cudaEventCreateWithFlags(&m->ev_join[i], cudaEventDisableTiming);
    if (e != cudaSuccess) {
        model_destroy(m);
        return set_cuda_error(e, "model_create: streams");
    }
    *out = m;
    return ARC_OK;
}

int model_set_layer(arcllm_cuda_model* m, uint32_t layer, const arcllm_cuda_layer* L) {
    if (!m || !L) return set_error(ARC_E_INVALID_ARGUMENT, "model_set_layer: null pointer");
    if (layer >= m->cfg.n_layers) return set_error(ARC_E_INVALID_ARGUMENT, "model_set_layer: layer out of range");
    ARC_TRY(check_layer(m->cfg, *L));
    m->layers[layer] = *L;
    m->layer_set[layer] = 1;
    // captured step graphs hold the previous weight pointers: re-capture on next use
    if (m->g_prefill) {
        cudaGraphExecDestroy(m->g_prefill);
        m->g_prefill = nullptr;
    }
    if (m->g_decode) {
        cudaGraphExecDestroy(m->g_decode);
        m->g_decode = nullptr;
    }
    return ARC_OK;
}

int model_set_endpoints(arcllm_cuda_model* m, const void* tok_embd, int tok_embd_type, const float* out_norm,
                        const void* out_w, int out_type) {
    if (!m || !tok_embd || !out_norm || !out_w) return set_error(ARC_E_INVALID_ARGUMENT, "set_endpoints: null pointer");
    if ((tok_embd_type != ARC_GGML_F16 && tok_embd_type != ARC_GGML_Q4_K) || !quant_ok(out_type))
        return set_error(ARC_E_UNSUPPORTED_SHAPE, "set_endpoints: embedding F16/Q4_K, output Q4_K/Q6_K");
    m->tok_embd = tok_embd;
    m->tok_embd_type = tok_embd_type;
    m->out_norm = out_norm;
    m->out_w = out_w;
    m->out_type = out_type;
    m->endpoints_set = true;
    return ARC_OK;
}

int model_tp_exchange_words(const arcllm_cuda_model_config* cfg, uint32_t n_ranks, uint32_t* out) {
    if (!cfg || !out || n_ranks == 0 || n_ranks > 8) return set_error(ARC_E_INVALID_ARGUMENT, "tp words: bad argument");
    *out = std::max(n_ranks * cfg->hidden, 4u * n_ranks);  // the partials of every rank; the greedy records
    return ARC_OK;
}

int model_set_tensor_parallel(arcllm_cuda_model* m, void* const* rank_bufs, uint32_t n_ranks, uint32_t rank,
                              uint32_t timeout_us) {
    if (!m || n_ranks == 0 || n_ranks > 8 || rank >= n_ranks || (n_ranks > 1 && !rank_bufs))
        return set_error(ARC_E_INVALID_ARGUMENT, "tensor parallel: 1..8 ranks, rank < n_ranks, buffers");
    const arcllm_cuda_model_config& c = m->cfg;
    ExchangeRanks tp{};
    uint32_t fr0 = 0, frows = c.ffn, lr0 = 0, lrows = c.vocab;
    if (n_ranks > 1) {
        // s in whole pairs of super-blocks (512 rows): a K window of the Q6_K down projection
        // must start and end on an even block
        if (c.ffn % kTpFfnAlign || c.vocab % kTpRowAlign || c.hidden % 4u)
            return set_error(ARC_E_UNSUPPORTED_SHAPE, "tensor parallel: ffn % 512 == 0, vocab % 32 == 0");
        ARC_TRY(shard_rows(c.ffn, kTpFfnAlign, n_ranks, rank, &fr0, &frows));
        ARC_TRY(shard_rows(c.vocab, kTpRowAlign, n_ranks, rank, &lr0, &lrows));
        uint32_t words = 0;
        ARC_TRY(model_tp_exchange_words(&c, n_ranks, &words));
        for (uint32_t q = 0; q < n_ranks; ++q) {
            if (!rank_bufs[q] || (reinterpret_cast<uintptr_t>(rank_bufs[q]) & 255u))
                return set_error(ARC_E_ALIGNMENT, "tensor parallel: rank buffers must be 256-byte aligned");
            tp.bufs[q] = rank_bufs[q];
        }
        tp.n_ranks = n_ranks;
        tp.rank = rank;
        tp.max_words = words;
        tp.timeout_us = timeout_us;
        if (!m->tp_part) {
            void* p = nullptr;
            const cudaError_t e = cudaMalloc(&p, 4ull * c.hidden + 256u);
            if (e != cudaSuccess) return set_cuda_error(e, "tensor parallel: partial sums and greedy records");
            m->tp_part = static_cast<float*>(p);
            m->tp_recs = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(p) + 4ull * c.hidden);
        }
        // split-K scratch for the down projection's K window, before any graph capture
        const int down_types[3] = {ARC_GGML_Q4_K, ARC_GGML_Q6_K, ARC_TYPE_EXEC148};
        for (int t : down_types) ARC_TRY(matvec_kwindow_reserve(t, c.hidden, frows / 256u));
    }
    m->tp = tp;
    m->ffn_r0 = fr0, m->ffn_rows = frows;
    m->lm_row0 = lr0, m->lm_rows = lrows;
    // the captured step graphs hold the previous layout: re-capture on next use
    if (m->g_prefill) {
        cudaGraphExecDestroy(m->g_prefill);
        m->g_prefill = nullptr;
    }
    if (m->g_decode) {
        cudaGraphExecDestroy(m->g_decode);
        m->g_decode = nullptr;
    }
    return ARC_OK;
}

int model_shard_lm_head(arcllm_cuda_model* m, uint32_t row0, uint32_t rows) {
    if (!m || rows == 0 || row0 + rows > m->cfg.vocab) return set_error(ARC_E_INVALID_ARGUMENT, "shard: bad range");
    m->lm_row0 = row0;
    m->lm_rows = rows;
    if (m->g_decode) {
        cudaGraphExecDestroy(m->g_decode);
        m->g_decode = nullptr;
    }
    return ARC_OK;
}

static int ready(arcllm_cuda_model* m) {
    if (!m->endpoints_set) return set_error(ARC_E_INVALID_ARGUMENT, "model: endpoints not set");
    for (uint8_t f : m->layer_set)
        if (!f) return set_error(ARC_E_INVALID_ARGUMENT, "model: not every layer was set");
    return ARC_OK;
}

int model_begin(arcllm_cuda_model* m, const uint32_t* prompt_host, uint32_t n_prompt, uint32_t max_new,
                cudaStream_t st) {
    if (!m || !prompt_host) return set_error(ARC_E_INVALID_ARGUMENT, "begin: null pointer");
    ARC_TRY(ready(m));
    if (n_prompt == 0 || max_new == 0) return set_error(ARC_E_INVALID_ARGUMENT, "begin: empty prompt or max_new 0");
    if ((uint64_t)n_prompt + max_new - 1u > m->cfg.max_ctx)
        return set_error(ARC_E_INVALID_ARGUMENT, "begin: request exceeds the KV context limit");
    for (uint32_t i = 0; i < n_prompt; ++i)
        if (prompt_host[i] >= m->cfg.vocab) return set_error(ARC_E_INVALID_ARGUMENT, "begin: token out of vocabulary");
    GreedyState s{};
    s.token = prompt_host[0];
    s.pos = 0;
    s.n_prompt = n_prompt;
    cudaError_t e = cudaMemcpyAsync(m->prompt, prompt_host, 4ull * n_prompt, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->state, &s, sizeof s, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);  // `s` lives on this stack frame
    if (e != cudaSuccess) return set_cuda_error(e, "begin: upload");
    m->begun_prompt = n_prompt;
    return ARC_OK;
}

// Prompt tokens 0 .. n-2 of the request begun last: batched on the tensor
// cores when the model allows it (else one fp32 prefill step per token).
// Afterwards the next step(with_head) yields the first generated token.
int model_prefill(arcllm_cuda_model* m, cudaStream_t st, bool* batched_out) {
    if (!m) return set_error(ARC_E_INVALID_ARGUMENT, "prefill: null model");
    ARC_TRY(ready(m));
    const uint32_t n_prompt = m->begun_prompt;
    if (n_prompt == 0) return set_error(ARC_E_INVALID_ARGUMENT, "prefill: begin() first");
    m->begun_prompt = 0;  // the prompt is consumed once
    const bool batched = n_prompt > 1 && prefill_batched_ok(m);
    m->launches_prefill_batched = 0;
    if (batched) {
        ARC_TRY(prefill_alloc(m));
        for (uint32_t p0 = 0; p0 + 1 < n_prompt; p0 += kPrefillRows)
            ARC_TRY(enqueue_prefill_chunk(m, p0, std::min(kPrefillRows, n_prompt - 1u - p0), st,
                                          &m->launches_prefill_batched));
        ARC_TRY(launch_prefill_done(m->state, m->prompt, n_prompt, st));
        ++m->launches_prefill_batched;
    } else {
        for (uint32_t i = 0; i + 1 < n_prompt; ++i) ARC_TRY(model_step(m, 0, 1, st));
    }
    if (batched_out) *batched_out = batched;
    return ARC_OK;
}

int model_step(arcllm_cuda_model* m, int with_head, int use_graph, cudaStream_t st) {
    if (!m) return set_error(ARC_E_INVALID_ARGUMENT, "step: null model");
    ARC_TRY(ready(m));
    if (!use_graph) return enqueue_step(m, with_head != 0, st, nullptr);
    cudaGraphExec_t* g = with_head ? &m->g_decode : &m->g_prefill;
    if (!*g) {
        ARC_TRY(capture(m, with_head != 0, g, with_head ? &m->launches_decode_step : &m->launches_prefill_step));
    }
    const cudaError_t e = cudaGraphLaunch(*g, st);
    return e == cudaSuccess ? ARC_OK : set_cuda_error(e, "graph launch");
}

int model_generate(arcllm_cuda_model* m, const uint32_t* prompt_host, uint32_t n_prompt, uint32_t max_new,
                   uint32_t* out_host, arcllm_cuda_gen_stats* stats, cudaStream_t st) {
    if (!out_host) return set_error(ARC_E_INVALID_ARGUMENT, "generate: null output");
    ARC_TRY(model_begin(m, prompt_host, n_prompt, max_new, st));
    // make sure both graphs exist before timing (capture is host work)
    if (!m->g_prefill) ARC_TRY(capture(m, false, &m->g_prefill, &m->launches_prefill_step));
    if (!m->g_decode) ARC_TRY(capture(m, true, &m->g_decode, &m->launches_decode_step));
    cudaEvent_t e0, e1, e2;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventCreate(&e2);
    if (n_prompt > 1 && prefill_batched_ok(m)) ARC_TRY(prefill_alloc(m));  // outside the timed region
    bool batched = false;
    cudaEventRecord(e0, st);
    ARC_TRY(model_prefill(m, st, &batched));
    ARC_TRY(model_step(m, 1, 1, st));  // last prompt token: first generated token
    cudaEventRecord(e1, st);
    for (uint32_t i = 1; i < max_new; ++i) ARC_TRY(model_step(m, 1, 1, st));
    cudaEventRecord(e2, st);
    GreedyState s{};
    cudaError_t e = cudaMemcpyAsync(out_host, m->out_tokens, 4ull * max_new, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(&s, m->state, sizeof s, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    float ms_p = 0.f, ms_d = 0.f;
    if (e == cudaSuccess) {
        cudaEventElapsedTime(&ms_p, e0, e1);
        cudaEventElapsedTime(&ms_d, e1, e2);
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaEventDestroy(e2);
    if (e != cudaSuccess) return set_cuda_error(e, "generate: readback");
    if (stats) {
        if (batched) {
            stats->prefill_launches = m->launches_prefill_batched + m->launches_decode_step;
            stats->prefill_graph_launches = 1;
        } else {
            stats->prefill_launches = m->launches_prefill_step * (n_prompt - 1u) + m->launches_decode_step;
            stats->prefill_graph_launches = n_prompt;
        }
        stats->decode_launches_per_step = m->launches_decode_step;
        stats->decode_graph_launches_per_step = 1;
        stats->decode_steps = max_new - 1u;
        stats->prefill_ms = ms_p;
        stats->decode_ms = ms_d;
        stats->finite = (s.nonfinite == 0) ? 1 : 0;
    }
    if (s.n_generated != max_new) return set_error(ARC_E_INVALID_ARGUMENT, "generate: generated-token count mismatch");
    if (s.nonfinite) return set_error(ARC_E_NONFINITE, "generate: non-finite logits");
    return ARC_OK;
}

int model_set_prefill_mode(arcllm_cuda_model* m, int mode) {
    if (!m || (mode != 0 && mode != 1)) return set_error(ARC_E_INVALID_ARGUMENT, "prefill mode: 0 or 1");
    m->prefill_mode = mode;
    return ARC_OK;
}

int model_set_prefill_down(arcllm_cuda_model* m, uint32_t layer, const void* w, int type) {
    if (!m || !w) return set_error(ARC_E_INVALID_ARGUMENT, "prefill down: null pointer");
    if (layer >= m->cfg.n_layers) return set_error(ARC_E_INVALID_ARGUMENT, "prefill down: layer out of range");
    if (!quant_ok(type)) return set_error(ARC_E_UNSUPPORTED_SHAPE, "prefill down: Q4_K or Q6_K");
    m->prefill_down[layer] = w;
    m->prefill_down_type[layer] = type;
    return ARC_OK;
}

int model_logits(arcllm_cuda_model* m, const float** out) {
    if (!m || !out) return set_error(ARC_E_INVALID_ARGUMENT, "logits: null pointer");
    *out = m->logits;
    return ARC_OK;
}

int model_kv_cache(arcllm_cuda_model* m, const uint16_t** k, const uint16_t** v) {
    if (!m || !k || !v) return set_error(ARC_E_INVALID_ARGUMENT, "kv_cache: null pointer");
    *k = m->kc;
    *v = m->vc;
    return ARC_OK;
}

int model_destroy(arcllm_cuda_model* m) {
    if (!m) return ARC_OK;
    if (m->g_prefill) cudaGraphExecDestroy(m->g_prefill);
    if (m->g_decode) cudaGraphExecDestroy(m->g_decode);
    if (m->arena) cudaFree(m->arena);
    if (m->pf_arena) cudaFree(m->pf_arena);
    if (m->tp_part) cudaFree(m->tp_part);
    for (int i = 0; i < 2; ++i) {
        if (m->side[i]) cudaStreamDestroy(m->side[i]);
        if (m->ev_join[i]) cudaEventDestroy(m->ev_join[i]);
    }
    if (m->ev_fork) cudaEventDestroy(m->ev_fork);
    delete m;
    return ARC_OK;
}

}  // namespace arc
