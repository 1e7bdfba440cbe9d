// Internal declarations shared by the CUDA translation units of
// libarcllm_cuda.so.  Nothing here crosses the C ABI (include/arcllm_cuda.h).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "../../include/arcllm_cuda.h"

namespace arc {

// Record a status + message for arcllm_cuda_last_error_message(); returns status.
int set_error(int status, const char* msg);
int set_cuda_error(cudaError_t e, const char* where);

// Index of the current device in the library's per-device tables (64 slots); -1 when there is no
// current device or its index is 64 or more (such devices are not supported).
inline int device_slot() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
    return dev;
}

// Device address of this library's device error word on the current device
// (nullptr if it cannot be resolved).
unsigned int* dev_error_word();

// Programmatic dependent launch (PDL).  While a PdlScope is active on this
// thread, kernels are launched with programmatic stream serialization: the
// next kernel may start while the previous one drains, every kernel waits
// (griddepcontrol.wait) before touching its predecessors' outputs, and the
// matvecs stream their weights before that wait.  Only code whose weights are
// not written by the preceding kernels may enable it (the model's decode
// graphs); ARCLLM_PDL=0 disables it.
bool pdl_enabled();
class PdlScope {
public:
    explicit PdlScope(bool on);
    ~PdlScope();
private:
    bool prev_;
};

template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    if (pdl_enabled()) {
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
    return e != cudaSuccess ? e : cudaGetLastError();
}

struct MatvecPlan {
    int fmt = 0;
    bool dual = false;
    bool xreg = false;  // x held in registers (one 32-weight unit per consumer thread)
    uint32_t nwc = 0;   // consumer warps per CTA
    uint32_t rows = 0, k = 0, nb = 0, rb = 0;
    uint32_t G = 0, gmax = 0, n_groups = 0, stages = 0, stage_smem = 0, x_floats = 0;
    uint32_t smem = 0, grid = 0;
};

// Load and configure every matvec kernel on the current device (idempotent);
// call before capturing launches into a CUDA graph.
int matvec_prepare();
int matvec_plan(int fmt, bool dual, uint32_t rows, uint32_t k, MatvecPlan* out);
// Integer tensor-core variant (matvec_imma.cu), K/256 <= 14 (even for Q6_K).
int matvec_imma_prepare();
bool matvec_imma_supported(int fmt, bool dual, uint32_t rows, uint32_t k);
// Fused RoPE / KV-store epilogue of the whole-row kernel (mode 1: rotate rows in pairs at
// position *pos and write y; 2: also store fp16 to cache row *pos; 3: store fp16 unrotated).
struct RopeEpilogue {
    uint32_t mode, half, max_ctx;
    const float2* table;
    const uint32_t* pos;
    uint16_t* cache;  // this layer's cache: row p at p * rows
};
// Rank all-gather epilogue of the whole-row kernel (fence-free): each row of this rank's shard
// [row0, row0 + rows) goes to every rank r as one 64-bit word (epoch << 32 | fp32 bits) at
// ll[r][row0 + i] (ll[r]: rank r's word array of rows_total words, an NVLink peer mapping for
// r != self_rank); the launch ends once this rank's words all carry `epoch`, their values copied
// to out[0, rows_total).
struct RankGather {
    uint32_t n_ranks, self_rank, epoch, row0, rows_total;
    unsigned long long wait_ns;
    unsigned long long* ll[8];
    float* out;
};
// One job of matvec_imma_multi_launch: y = W . RMSNorm(x) (+ bias, RoPE / KV-store epilogue).
struct ImmaJob {
    int fmt;
    const void* w;
    uint32_t rows;
    const float* bias;
    float* y;
    const RopeEpilogue* rope;
};
// The decode step's Q, K and V projections (same x, gamma and K) as ONE launch, each job on its
// own CTAs; supported when every job takes the whole-row kernel with 32-row groups and all the
// groups fit on the SMs at once.
bool matvec_imma_multi_supported(const ImmaJob (&jobs)[3], uint32_t k);
int matvec_imma_multi_launch(const ImmaJob (&jobs)[3], uint32_t k, const float* x, const float* gamma, float eps,
                             cudaStream_t stream);
int matvec_imma_launch(int fmt, bool dual, const void* w0, const void* w1, uint32_t rows, uint32_t k, const float* x,
                       const float* gamma, float eps, const float* bias, const float* residual, float* y,
                       cudaStream_t stream, const RopeEpilogue* rope = nullptr, const RankGather* gather = nullptr);
// Integer tensor-core K-slice variant (matvec_imma_splitk.cu) for K > 3584.
// It adds CTA partials through a per-device scratch: launches of it on one
// device must not overlap in time (one stream, or ordered streams).
// matvec_splitk_reserve sizes that scratch ahead of graph capture.
int matvec_splitk_prepare();
int matvec_splitk_reserve(int fmt, uint32_t rows, uint32_t k);
bool matvec_splitk_supported(int fmt, bool dual, uint32_t rows, uint32_t k);
int matvec_splitk_launch(int fmt, const void* w, uint32_t rows, uint32_t k, const float* x, const float* gamma,
                         float eps, const float* bias, const float* residual, float* y, cudaStream_t stream);
// The K-slice kernel over super-blocks [kb_base, kb_base + nb_win) of every row (x indexed by
// the full K; no RMSNorm): the tensor-parallel FFN down projection of a rank's slice of s.
int matvec_kwindow_launch(int fmt, const void* w, uint32_t rows, uint32_t k, uint32_t kb_base, uint32_t nb_win,
                          const float* x, const float* gamma, float eps, const float* bias, const float* residual,
                          float* y, cudaStream_t stream);
int matvec_kwindow_reserve(int fmt, uint32_t rows, uint32_t nb_win);
// Pick the kernel for a matvec: the integer tensor-core forms where they
// apply (whole rows for K <= 3584, K slices for K > 3584), else the CUDA-core
// streaming form (ARCLLM_MATVEC_IMPL=cuda forces the CUDA-core form).
int matvec_any(int fmt, bool dual, const void* w0, const void* w1, uint32_t rows, uint32_t k, const float* x,
               const float* gamma, float eps, const float* bias, const float* residual, float* y,
               cudaStream_t stream);
int matvec_launch(const MatvecPlan& pl, const void* w0, const void* w1, const float* x, const float* gamma,
                  float eps, const float* bias, const float* residual, float* y, cudaStream_t stream);

// Rank exchange over NVLink peer stores (exchange.cu).  bufs[q]: rank q's
// exchange buffer as this process maps it (its own allocation for q == rank),
// exchange_buffer_bytes(max_words) bytes, 256-byte aligned, zero-filled once.
struct ExchangeRanks {
    void* bufs[8];
    uint32_t n_ranks, rank, max_words, timeout_us;
};
uint64_t exchange_buffer_bytes(uint32_t max_words);
// dst[0, n_total) on every rank = the slices src[0, n_local) that each rank
// contributes at its offset `off` (32-bit words).
int exchange_gather(const ExchangeRanks& ex, const void* src, uint32_t n_local, uint32_t off, void* dst,
                    uint32_t n_total, cudaStream_t stream);
// dst[i] = residual[i] (nullable) + sum over ranks r (in rank order) of rank r's src[i], i < n,
// on every rank; needs n_ranks * n <= max_words.
int exchange_reduce(const ExchangeRanks& ex, const float* src, uint32_t n, const float* residual, float* dst,
                    cudaStream_t stream);
int shard_rows(uint32_t n, uint32_t align, uint32_t n_ranks, uint32_t rank, uint32_t* row0, uint32_t* rows);

// cuTensorMapEncodeTiled (driver entry point), or null (gemm_tcgen05.cu).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled_fn();

// EXEC148 image of Q4_K weights (exec148.cu).
int exec148_materialize(const void* src, uint64_t n_blocks, void* dst, cudaStream_t stream);
int exec148_validate(const void* src, const void* img, uint64_t n_blocks, uint64_t* mismatches_host,
                     cudaStream_t stream);
int exec148_matvec(const void* w, uint32_t rows, uint32_t k, const float* x, const float* residual, float* y,
                   cudaStream_t stream);

// Prefill GEMM on tcgen05 (gemm_tcgen05.cu).
int gemm_q4k_bf16_prepare();
int gemm_q4k_bf16(const void* w, uint32_t n, uint32_t k, const uint16_t* x, uint32_t m, float* y,
                  cudaStream_t stream);
// Q4_K (12) or Q6_K (14) weights; y = residual + x W^T when residual is non-null.
// mode 0: x and the dequantised W in bf16; 1: both fp16 (x holds fp16);
// 2: fp16 hi + lo of both, y = (x + x_lo)(W_hi + W_lo)^T without the lo*lo term.
int gemm_kq_bf16(int fmt, const void* w, uint32_t n, uint32_t k, const uint16_t* x, uint32_t m,
                 const float* residual, float* y, cudaStream_t stream, int mode = 0, const uint16_t* x_lo = nullptr);
// Output-row-sharded GEMM with the result all-gathered by its reduce kernel over NVLink peer stores:
// this rank's columns [c0, c0 + n) of an m x n_total result into every rank's buffer (rank_bufs,
// gemm_gather_flags_offset(m, n_total) + 128 bytes each, zeroed before first use), then a flag handshake.
uint64_t gemm_gather_flags_offset(uint32_t m, uint32_t n_total);
int gemm_kq_allgather(int fmt, const void* w, uint32_t n, uint32_t k, const uint16_t* x, uint32_t m, uint32_t c0,
                      uint32_t n_total, void* const* rank_bufs, uint32_t n_ranks, uint32_t rank, uint32_t epoch,
                      uint32_t timeout_us, cudaStream_t stream);

std::vector<float> rope_table(uint32_t max_ctx, uint32_t head_dim, float theta);
int model_create(const arcllm_cuda_model_config* cfg, arcllm_cuda_model** out);
int model_destroy(arcllm_cuda_model* m);
int model_set_layer(arcllm_cuda_model* m, uint32_t layer, const arcllm_cuda_layer* L);
int model_set_endpoints(arcllm_cuda_model* m, const void* tok_embd, int tok_embd_type, const float* out_norm,
                        const void* out_w, int out_type);
int model_shard_lm_head(arcllm_cuda_model* m, uint32_t row0, uint32_t rows);
int model_begin(arcllm_cuda_model* m, const uint32_t* prompt_host, uint32_t n_prompt, uint32_t max_new,
                cudaStream_t st);
int model_step(arcllm_cuda_model* m, int with_head, int use_graph, cudaStream_t st);
int model_prefill(arcllm_cuda_model* m, cudaStream_t st, bool* batched_out);
int model_tp_exchange_words(const arcllm_cuda_model_config* cfg, uint32_t n_ranks, uint32_t* out);
int model_set_tensor_parallel(arcllm_cuda_model* m, void* const* rank_bufs, uint32_t n_ranks, uint32_t rank,
                              uint32_t timeout_us);
int model_generate(arcllm_cuda_model* m, const uint32_t* prompt_host, uint32_t n_prompt, uint32_t max_new,
                   uint32_t* out_host, arcllm_cuda_gen_stats* stats, cudaStream_t st);
int model_set_prefill_mode(arcllm_cuda_model* m, int mode);
int model_set_prefill_down(arcllm_cuda_model* m, uint32_t layer, const void* w, int type);
int model_logits(arcllm_cuda_model* m, const float** out);
int model_kv_cache(arcllm_cuda_model* m, const uint16_t** k, const uint16_t** v);

}  // namespace arc
