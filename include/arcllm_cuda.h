/*
 * arcllm_cuda.h -- C ABI of libarcllm_cuda.so, the B200 (sm_100a) kernels behind
 * ArcLLM's decode hot path.
 *
 * Conventions
 *   - Every entry point returns an int status (ARC_OK == 0).  Nothing throws
 *     across this boundary.  arcllm_cuda_last_error_message() gives the detail
 *     of the last failure on the calling thread.
 *   - Pointers named w, x, y, ... are DEVICE pointers unless the name says
 *     `host`.  `stream` is a cudaStream_t passed as void* (NULL = legacy
 *     default stream).  Launches are asynchronous.
 *   - Quantised weights are GGUF row-major tensors of super-blocks:
 *       Q4_K (ggml type 12): 256 weights in 144 bytes
 *                            {fp16 d, fp16 dmin, 12 B scales/mins, 128 B nibbles}
 *       Q6_K (ggml type 14): 256 weights in 210 bytes
 *                            {128 B ql, 64 B qh, 16 x int8 scales, fp16 d}
 *     A row of K weights is K/256 consecutive super-blocks.  Weight pointers
 *     must be 16-byte aligned (the matvec streams them with TMA bulk copies).
 *   - Activations are fp32.
 *
 * Each declaration names the reference interface it replaces (paths relative
 * to the ArcLLM repository root).  The reference has no C ABI of its own: its
 * runtime records Vulkan dispatches with push-constant structs declared at
 * src/arcllm_v1_runtime.cpp:268-277, which is what these functions take over.
 */
#ifndef ARCLLM_CUDA_H
#define ARCLLM_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ARCLLM_CUDA_ABI_VERSION 1

#if defined(__GNUC__)
#define ARCLLM_CUDA_API __attribute__((visibility("default")))
#else
#define ARCLLM_CUDA_API
#endif

enum arcllm_cuda_status {
    ARC_OK = 0,
    ARC_E_INVALID_ARGUMENT = 1,  /* null pointer, zero size, bad format id     */
    ARC_E_ALIGNMENT = 2,         /* pointer not aligned as documented          */
    ARC_E_UNSUPPORTED_SHAPE = 3, /* shape outside what the kernels implement   */
    ARC_E_CUDA = 4,              /* CUDA runtime error (see last_error_message) */
    ARC_E_OUT_OF_MEMORY = 5,
    ARC_E_DEVICE_TIMEOUT = 6,    /* a bounded device-side wait gave up         */
    ARC_E_NONFINITE = 7,         /* non-finite logits (reference: runtime.cpp:446,501) */
    ARC_E_NCCL = 8
};

enum arcllm_ggml_type { ARC_GGML_F32 = 0, ARC_GGML_F16 = 1, ARC_GGML_Q4_K = 12, ARC_GGML_Q6_K = 14 };
/* Not a GGUF type: the EXEC148 image of a Q4_K matrix (primitive B of the
 * Q4 FFN-down capability, src/q4_down_exec148_materializer.h:14), 148 bytes
 * per super-block.  Accepted by arcllm_cuda_matvec (without gamma or bias)
 * and as a layer's type_down. */
enum { ARC_TYPE_EXEC148 = 148 };

ARCLLM_CUDA_API int arcllm_cuda_abi_version(void);
ARCLLM_CUDA_API const char *arcllm_cuda_status_string(int status);
ARCLLM_CUDA_API const char *arcllm_cuda_last_error_message(void);

/* Reads (and clears) the device error word the kernels set when a bounded
 * wait gives up (bit 0), an index check fails (bit 1) or an fp16 operand
 * leaves the fp16 range (bit 2).  Synchronises
 * `stream` first.  Returns ARC_E_DEVICE_TIMEOUT if bit 0 was set. */
ARCLLM_CUDA_API int arcllm_cuda_device_error(void *stream, uint32_t *out_bits);

/* ---- bit-exact dequantisation -------------------------------------------
 * y[i*256 + k] = value of element k of super-block i, computed exactly as
 * src/p8c_segmented_access_correctness.cpp:1166-1181 (Q4_K, q4k_dequant_row_p8c)
 * and :944-956 (Q6_K, q6k_dequant_row): d*sc*q - dmin*mn with separately
 * rounded fp32 operations. */
ARCLLM_CUDA_API int arcllm_cuda_dequant_q4k(const void *w, uint64_t n_blocks, float *y, void *stream);
ARCLLM_CUDA_API int arcllm_cuda_dequant_q6k(const void *w, uint64_t n_blocks, float *y, void *stream);

/* ---- M = 1 dequant-matvec ------------------------------------------------
 * y[r] = residual[r] + bias[r] + sum_k W[r,k] * xn[k],   r < rows
 * with xn = x, or xn = rmsnorm(x) * gamma when gamma != NULL (eps as given).
 * bias, residual and gamma may be NULL; y must not alias x or W.
 * Replaces: shaders/p7_q4k_gemm_2d.comp and shaders/p7_q6k_gemm_2d.comp with
 * push constants PCGemm{n=k, rows, batch=1, row_bytes, add_bias, w_base, bias_base}
 * (src/arcllm_v1_runtime.cpp:270, decode use :380-387, :410-413);
 * shaders/sa1_q4k_subgroup_splitk.comp (I002 gate/up and FFN-down route A,
 * src/arcllm_v1_runtime.cpp:390-396, src/arcllm_v1_q4_vulkan_backend_v4_runtime.h:357-366);
 * shaders/p8q1_lmhead_q6k_segmented_chunk.comp (LM head, PCLMSeg,
 * src/arcllm_v1_runtime.cpp:277,285-291); the fused RMSNorm replaces
 * shaders/p7_rmsnorm_seq.comp (PCRms, :271) and the residual replaces
 * shaders/p7_add.comp (PCN, :276).  k must be a multiple of 256, <= 32768.
 * Row sharding: pass w advanced by r0*row_bytes (keep 16-byte alignment) and
 * y advanced by r0. */
ARCLLM_CUDA_API int arcllm_cuda_matvec(int ggml_type, const void *w, uint32_t rows, uint32_t k, const float *x,
                       const float *gamma, float eps, const float *bias, const float *residual, float *y,
                       void *stream);
ARCLLM_CUDA_API int arcllm_cuda_matvec_q4k(const void *w, uint32_t rows, uint32_t k, const float *x, const float *bias,
                           float *y, void *stream);
ARCLLM_CUDA_API int arcllm_cuda_matvec_q6k(const void *w, uint32_t rows, uint32_t k, const float *x, const float *bias,
                           float *y, void *stream);

/* End-to-end form for callers that hold HOST activations (the reference's
 * flow: input written to mapped memory, one submit, fence wait, logits read
 * back -- src/arcllm_v1_runtime.cpp:440-446):  copies k floats x_host ->
 * x_dev, runs arcllm_cuda_matvec (no norm/bias/residual), delivers the rows
 * floats to y_host and waits for `stream`.  x_dev / y_dev are caller-owned
 * device buffers.  A pinned (page-locked, hence device-mapped) y_host is
 * written by the kernel itself while it runs, as the reference reads logits
 * from host-visible mapped memory; a pageable y_host gets y_dev copied to it
 * after the kernel.  x_host should be pinned for an asynchronous copy. */
ARCLLM_CUDA_API int arcllm_cuda_matvec_hostio(int ggml_type, const void *w, uint32_t rows, uint32_t k,
                                              const float *x_host, float *x_dev, float *y_dev, float *y_host,
                                              void *stream);

/* ---- row-sharded matvec with the result all-gathered over NVLink --------
 * Multi-GPU form of the LM head (rows sharded over the ranks: rank r owns rows
 * [row0, row0 + rows) of a rows_total-row matrix; the reference runs the LM
 * head on one device, src/arcllm_v1_runtime.cpp:285-291).  One kernel per
 * rank computes its rows and stores each result into EVERY rank's exchange
 * buffer as one 64-bit word (epoch << 32 | fp32 bits; a local store for its
 * own buffer, NVLink peer stores for the others); each launch then reads its
 * own buffer's words until all carry its epoch -- every word is its own flag,
 * so no fence or separate handshake is needed -- and copies the values into
 * its logits: when the launch completes on rank r, all rows_total logits are
 * at rank_bufs[r] + arcllm_cuda_allgather_logits_offset(rows_total).  This
 * replaces matvec + ncclAllGather.
 *   rank_bufs[i]: this process's device address of rank i's exchange buffer
 *                 (its own allocation for i == rank, an IPC mapping otherwise),
 *                 256-byte aligned, arcllm_cuda_allgather_buffer_bytes bytes,
 *                 zero-filled before first use; consecutive launches alternate
 *                 between two such buffer sets (epoch parity);
 *   epoch: 1, 2, 3 ... -- the same sequence on every rank, one per launch;
 *   timeout_us: bound of the wait for the other ranks' rows (0: 2 s); a wait
 *               that runs out sets the device error word (ARC_E_DEVICE_TIMEOUT
 *               via arcllm_cuda_device_error) and the kernel returns.
 * A rank may not rewrite a buffer that peers still store into: launches of
 * one epoch sequence must not overlap a reader of the previous logits.
 * Shapes: the whole-row tensor-core kernel (K/256 <= 14, even for Q6_K),
 * 16-byte aligned x; n_ranks <= 8. */
ARCLLM_CUDA_API int arcllm_cuda_allgather_buffer_bytes(uint32_t rows_total, uint64_t *out);
/* Byte offset of the gathered fp32 logits inside an exchange buffer. */
ARCLLM_CUDA_API int arcllm_cuda_allgather_logits_offset(uint32_t rows_total, uint64_t *out);
ARCLLM_CUDA_API int arcllm_cuda_matvec_allgather(int ggml_type, const void *w, uint32_t rows, uint32_t k,
                                                 const float *x, uint32_t row0, uint32_t rows_total,
                                                 void *const *rank_bufs, uint32_t n_ranks, uint32_t rank,
                                                 uint32_t epoch, uint32_t timeout_us, void *stream);
/* The same launch with host buffers (the multi-GPU form of
 * arcllm_cuda_matvec_hostio): copies x_host (k floats) into x_dev, runs the
 * all-gather matvec and returns once all rows_total logits are in y_host.
 * Pinned, device-mapped y_host: the kernel's collect phase stores every
 * logit straight into it over the host link (no copy after the kernel);
 * pageable y_host: one device-to-host copy of the gathered logits.  With a
 * pinned y_host the rank's own logits area holds only its own rows.
 * Synchronises `stream`. */
ARCLLM_CUDA_API int arcllm_cuda_matvec_allgather_hostio(int ggml_type, const void *w, uint32_t rows, uint32_t k,
                                                        const float *x_host, float *x_dev, uint32_t row0,
                                                        uint32_t rows_total, void *const *rank_bufs,
                                                        uint32_t n_ranks, uint32_t rank, uint32_t epoch,
                                                        uint32_t timeout_us, float *y_host, void *stream);
/* CUDA IPC of exchange buffers between the ranks' processes: a 64-byte
 * handle of a buffer allocated with arcllm_cuda_malloc, opened in a peer
 * process (peer access enabled lazily), closed before the owner frees it. */
ARCLLM_CUDA_API int arcllm_cuda_ipc_get_handle(const void *dev_ptr, void *handle_out);
ARCLLM_CUDA_API int arcllm_cuda_ipc_open_handle(const void *handle, void **dev_ptr_out);
ARCLLM_CUDA_API int arcllm_cuda_ipc_close_handle(void *dev_ptr);

/* ---- rank exchange (all-gather of a vector over NVLink peer stores) ------
 * Not in the reference (it decodes on one device, src/arcllm_v1_runtime.cpp:
 * 371-421); the reassembly step of row-sharded matvecs.  Each rank stores its
 * slice src[0, n_local) (32-bit words) at word `offset` of every rank's
 * exchange buffer, each word as one 64-bit word tagged with the exchange's
 * sequence number (NVLink peer stores; nothing reads another GPU's memory),
 * then reads the assembled vector dst[0, n_total) out of its own buffer,
 * waiting (bounded by timeout_us, 0: 2 s) until every word carries the
 * sequence number -- each word is its own flag, no fence or handshake.
 *   rank_bufs[q]: rank q's buffer as this process maps it (own allocation for
 *   q == rank, an IPC mapping otherwise), arcllm_cuda_exchange_buffer_bytes
 *   (max_words) bytes, 256-byte aligned, zero-filled before first use.
 * Every rank must issue the same sequence of exchanges (the sequence numbers
 * live in the buffers, so a CUDA graph of exchanges replays unchanged).  A
 * wait that runs out sets the device error word's timeout bit (ARC_E_DEVICE_
 * TIMEOUT from arcllm_cuda_device_error) and leaves the words that did not
 * arrive out of dst; the buffers must then be zeroed on every rank before
 * further use. */
ARCLLM_CUDA_API int arcllm_cuda_exchange_buffer_bytes(uint32_t max_words, uint64_t *out);
ARCLLM_CUDA_API int arcllm_cuda_exchange_gather(void *const *rank_bufs, uint32_t n_ranks, uint32_t rank,
                                                uint32_t max_words, const void *src, uint32_t n_local,
                                                uint32_t offset, void *dst, uint32_t n_total, uint32_t timeout_us,
                                                void *stream);
/* The contiguous row shard [*row0, *row0 + *rows) of n rows that `rank` of
 * n_ranks owns: whole units of `align` rows (n % align == 0), the remainder
 * units one each to the first ranks.  Host-only arithmetic. */
ARCLLM_CUDA_API int arcllm_cuda_shard_rows(uint32_t n, uint32_t align, uint32_t n_ranks, uint32_t rank,
                                           uint32_t *row0, uint32_t *rows);

/* ---- fused gate/up projection with SiLU-multiply (Q4_K) -------------------
 * s[r] = silu(g[r]) * u[r],  g = W_gate . xn,  u = W_up . xn,  xn as above.
 * Replaces the I002 pair of shaders/sa1_q4k_subgroup_splitk.comp dispatches
 * plus shaders/p7_swiglu.comp (src/arcllm_v1_runtime.cpp:390-405) and the
 * ffn_norm shaders/p7_rmsnorm_seq.comp before them (:389). */
ARCLLM_CUDA_API int arcllm_cuda_gateup_silu_q4k(const void *w_gate, const void *w_up, uint32_t rows, uint32_t k,
                                const float *x, const float *gamma, float eps, float *s, void *stream);

/* The decode FFN block (src/arcllm_v1_runtime.cpp:389-415: ffn_norm RMSNorm,
 * the gate/up pair, SwiGLU, the down projection, the residual add):
 *   s = silu(W_gate . xn) * (W_up . xn),  y = residual + W_down . s
 * with xn = RMSNorm(x) * gamma; gate/up Q4_K (ffn x hidden), down Q4_K or
 * Q6_K (hidden x ffn); residual may be null; s (ffn floats) is written too.
 * Two launches on the stream: arcllm_cuda_gateup_silu_q4k, then
 * arcllm_cuda_matvec of the down projection. */
ARCLLM_CUDA_API int arcllm_cuda_ffn_block(int down_type, const void *w_gate, const void *w_up, const void *w_down,
                                          uint32_t hidden, uint32_t ffn, const float *x, const float *gamma,
                                          float eps, float *s, const float *residual, float *y, void *stream);

/* EXEC148 image of n_blocks Q4_K super-blocks (src/q4_down_exec148_materializer.h:14,
 * shaders/b1_2_exec148_gpu_materialize.comp: acquisition path P1 on the GPU).
 * q4k 16-byte aligned, exec 4-byte aligned, exec holds 148 * n_blocks bytes. */
ARCLLM_CUDA_API int arcllm_cuda_exec148_materialize(const void *q4k, uint64_t n_blocks, void *exec, void *stream);
/* Identity validation of an EXEC148 image against its Q4_K source
 * (src/q4_down_exec148_materializer.h:16-18: canonical tuples d, dmin,
 * 8 x (sc, mn), 256 codes must be identical).  Synchronous; writes the number
 * of differing blocks (0 = exact) to *mismatches_host. */
ARCLLM_CUDA_API int arcllm_cuda_exec148_validate(const void *q4k, const void *exec, uint64_t n_blocks,
                                                 uint64_t *mismatches_host, void *stream);

/* Prefill GEMM (config 4) on the tcgen05 tensor cores: y[m][n] (fp32, row-major)
 * = x[m][k] (bf16, row-major) * W^T for the n x k Q4_K matrix W, weights
 * dequantised to bf16 in shared memory, fp32 accumulation in TMEM.  Replaces
 * the prefill kernels shaders/p7l_ffn_q4k_gateup_fused.comp:22-38 and
 * shaders/p7g_ffn_q4k_tiled16.comp:15-34 (PCGemm/PCFusedGU with batch = seq,
 * src/arcllm_v1_runtime.cpp:343-366).  1 <= m <= 256, n % 128 == 0,
 * k % 256 == 0; w, x, y 16-byte aligned. */
ARCLLM_CUDA_API int arcllm_cuda_gemm_q4k_bf16(const void *w, uint32_t n, uint32_t k, const uint16_t *x_bf16,
                                              uint32_t m, float *y, void *stream);

/* The same GEMM for Q4_K (type 12) or Q6_K (type 14) weights, with an
 * optional fp32 residual: y = residual + x * W^T when residual is non-null
 * (the residual adds of the prefill chain, src/arcllm_v1_runtime.cpp:343-366,
 * fused into the epilogue).  Q6_K rows need only be 2-byte aligned. */
ARCLLM_CUDA_API int arcllm_cuda_gemm_bf16(int type, const void *w, uint32_t n, uint32_t k, const uint16_t *x_bf16,
                                          uint32_t m, const float *residual, float *y, void *stream);
/* Output-row-sharded form of the same GEMM (config 4 over N GPUs; the
 * reference runs it on one device, src/arcllm_v1_runtime.cpp:343-366): rank
 * `rank` holds rows [c0, c0 + n) of the full n_total x k weight matrix (w
 * points at row c0) and computes those columns of y; the kernel that adds the
 * split-K partials stores every float4 of them into EVERY rank's m x n_total
 * result (its own with local stores, the others with NVLink peer stores --
 * stores only), then the ranks meet on per-rank flags: when the launch
 * completes on rank r, rank_bufs[r] holds all n_total columns.  This replaces
 * GEMM + ncclAllGather.
 *   rank_bufs[q]: rank q's buffer as this process maps it (IPC mapping for
 *   q != rank), arcllm_cuda_gemm_allgather_buffer_bytes(m, n_total) bytes,
 *   256-byte aligned, zero-filled before first use; consecutive launches
 *   alternate between two buffer sets (epoch parity), as for
 *   arcllm_cuda_matvec_allgather;
 *   epoch: 1, 2, 3 ... the same sequence on every rank; timeout_us bounds the
 *   flag wait (0: 2 s; a wait that runs out sets the device error word).
 * c0 and n_total multiples of 4, n % 128 == 0; bf16 operands (mode 0). */
ARCLLM_CUDA_API int arcllm_cuda_gemm_allgather_buffer_bytes(uint32_t m, uint32_t n_total, uint64_t *out);
ARCLLM_CUDA_API int arcllm_cuda_gemm_bf16_allgather(int type, const void *w, uint32_t n, uint32_t k,
                                                    const uint16_t *x_bf16, uint32_t m, uint32_t c0,
                                                    uint32_t n_total, void *const *rank_bufs, uint32_t n_ranks,
                                                    uint32_t rank, uint32_t epoch, uint32_t timeout_us,
                                                    void *stream);
/* The same GEMM with fp16 operands: x_f16 is fp16 and the weights are
 * dequantised to fp16 (scale and offset of each sub-block and q*f - o rounded
 * to 11 significant bits instead of bf16's 8), at the same tensor-core rate.
 * generate() uses it for the prefill Q/K/V projections
 * (src/arcllm_v1_runtime.cpp:349-353), whose outputs feed the attention
 * scores: with bf16 operands the per-sub-block rounding of the scales moved
 * near-tied positions of the synthetic 7B-shape models.  Activations must stay
 * inside the fp16 range (|x| < 65504). */
ARCLLM_CUDA_API int arcllm_cuda_gemm_f16(int type, const void *w, uint32_t n, uint32_t k, const uint16_t *x_f16,
                                         uint32_t m, const float *residual, float *y, void *stream);
/* The same GEMM with ~22 significant bits of both operands: the activation as
 * fp16 halves x_hi = fp16(x), x_lo = fp16(x - x_hi), each weight dequantised
 * exactly in fp32 (as src/p8c_segmented_access_correctness.cpp:1166-1181 and
 * :944-956 do) and split into fp16 halves, y = residual + x_hi W_hi^T +
 * x_lo W_hi^T + x_hi W_lo^T (three MMAs per K step, fp32 accumulation).
 * generate() uses it for the prefill Q/K/V projections
 * (src/arcllm_v1_runtime.cpp:349-353): in the synthetic 7B-shape models the
 * attention scores run to 1e4, near-tied prompt positions are common over a
 * 255-row prompt, and one-operand fp16 rounding (~3.5e-4) moved whole cache
 * rows.  Same shapes and alignment as arcllm_cuda_gemm_bf16; |x| < 65504. */
ARCLLM_CUDA_API int arcllm_cuda_gemm_f16x3(int type, const void *w, uint32_t n, uint32_t k, const uint16_t *x_hi,
                                           const uint16_t *x_lo, uint32_t m, const float *residual, float *y,
                                           void *stream);
/* Batched RMSNorm of the prefill chain (shaders/p7_rmsnorm_seq.comp per row,
 * src/arcllm_v1_runtime.cpp:347,355; sum of squares in double as
 * src/p8c_segmented_access_correctness.cpp:958-969): out[r][i] = v rounded to
 * bf16 (out_fp16 == 0) or fp16, v = x[r][i] * rsqrt(mean(x[r]^2) + eps) * gamma[i];
 * with fp16 output and a non-null out_lo also out_lo[r][i] = fp16(v - out[r][i])
 * (the x_lo of arcllm_cuda_gemm_f16x3).  An fp16 value that overflows sets bit 2
 * of the device error word. */
ARCLLM_CUDA_API int arcllm_cuda_rmsnorm_rows(const float *x, const float *gamma, float eps, uint32_t rows, uint32_t h,
                                             int out_fp16, uint16_t *out, uint16_t *out_lo, void *stream);

/* ---- synthetic fixture streams -------------------------------------------
 * Deterministic, counter-based generators (element n of a splitmix64
 * sequence), identical bit for bit to the CPU test oracle, so multi-GB
 * synthetic models can be generated in HBM.  Not part of the reference
 * (its fixtures are host-side: src/sa1_component_benchmark.cpp:143-164). */
ARCLLM_CUDA_API int arcllm_cuda_fill_q4k(void *w, uint64_t block_begin, uint64_t n_blocks, uint64_t seed, void *stream);
ARCLLM_CUDA_API int arcllm_cuda_fill_q6k(void *w, uint64_t block_begin, uint64_t n_blocks, uint64_t seed, void *stream);
ARCLLM_CUDA_API int arcllm_cuda_fill_normal_f32(float *y, uint64_t begin, uint64_t n, uint64_t seed, float mu, float sigma,
                                void *stream);
ARCLLM_CUDA_API int arcllm_cuda_fill_normal_f16(uint16_t *y, uint64_t begin, uint64_t n, uint64_t seed, float mu, float sigma,
                                void *stream);


/* ---- decode-step ops (the model runs these; exposed for tests and callers
 * that drive their own step) ------------------------------------------------ */
/* Fill table[max_ctx][head_dim/2] with (cos, sin) of pos*theta^(-2p/head_dim),
 * evaluated in fp32 exactly as src/p8c_segmented_access_correctness.cpp:1010-1011.
 * Synchronous. */
ARCLLM_CUDA_API int arcllm_cuda_rope_table(float *table, uint32_t max_ctx, uint32_t head_dim, float theta);
/* RoPE on q [q_heads*head_dim] and k [kv_heads*head_dim] in place (adjacent
 * pairs, shaders/p7_rope_seq.comp:15-38, PCRope runtime.cpp:273) and store k, v
 * as fp16 into caches [layers][max_ctx][kv_heads*head_dim] at position *pos_dev
 * of `layer` (shaders/p7_kv_store.comp:14-25, PCKV runtime.cpp:274). */
ARCLLM_CUDA_API int arcllm_cuda_rope_kv_store(float *q, float *k, const float *v, const float *table,
                                              const uint32_t *pos_dev, uint16_t *k_cache, uint16_t *v_cache,
                                              uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
                                              uint32_t max_ctx, uint32_t layer, void *stream);
/* Cached GQA decode attention for position *pos_dev over fp16 caches
 * (shaders/p7_attention_kv_online.comp, PCAttnKV runtime.cpp:275; CPU form
 * src/p8c_segmented_access_correctness.cpp:1136-1158), split over n_splits
 * position slices per KV head.  head_dim must be 128.  `scratch` holds
 * kv_heads*n_splits*(q_heads/kv_heads)*(head_dim+2) floats. */
ARCLLM_CUDA_API int arcllm_cuda_attention_decode(const float *q, const uint16_t *k_cache, const uint16_t *v_cache,
                                                 const uint32_t *pos_dev, uint32_t q_heads, uint32_t kv_heads,
                                                 uint32_t head_dim, uint32_t max_ctx, uint32_t layer,
                                                 uint32_t n_splits, float *scratch, float *out, void *stream);
/* Batched prefill forms (the model's prefill chain; also for tests): rows t =
 * 0..rows-1 of q [rows][q_heads*head_dim], k and v [rows][kv_heads*head_dim]
 * get their biases (nullable) added, q and k the RoPE rotation of position
 * pos0+t (in place), and k, v are stored as fp16 at that position of `layer`;
 * then causal attention of query row t over cache positions 0..pos0+t, the
 * result written as bf16 [rows][q_heads*head_dim] (the O-projection GEMM's
 * operand).  head_dim must be 128; pos0+rows <= max_ctx. */
ARCLLM_CUDA_API int arcllm_cuda_rope_kv_rows(float *q, float *k, const float *v, const float *bq, const float *bk,
                                             const float *bv, const float *table, uint32_t pos0, uint32_t rows,
                                             uint16_t *k_cache, uint16_t *v_cache, uint32_t q_heads,
                                             uint32_t kv_heads, uint32_t head_dim, uint32_t max_ctx, uint32_t layer,
                                             void *stream);
ARCLLM_CUDA_API int arcllm_cuda_attention_prefill(const float *q, const uint16_t *k_cache, const uint16_t *v_cache,
                                                  uint32_t pos0, uint32_t rows, uint32_t q_heads, uint32_t kv_heads,
                                                  uint32_t head_dim, uint32_t max_ctx, uint32_t layer,
                                                  uint16_t *out_bf16, void *stream);
/* Same computation as arcllm_cuda_attention_decode, for callers that cannot
 * allocate device memory when they run a step (a host that fixes its device
 * memory plan in advance, a latency-critical loop that must not risk the
 * synchronisation cudaMalloc can cause, a plugin whose host owns the budget).
 * No counterpart in the reference.  The slice partials live in a 65536-float
 * (256 KiB) array inside the library, held on every GPU that loads it until
 * exit; needs kv_heads*n_splits*(q_heads/kv_heads)*(head_dim+2) <= 65536, else
 * ARC_E_UNSUPPORTED_SHAPE.  Allocates nothing.  All calls share the array:
 * calls that overlap on the GPU race; calls ordered on one stream are fine.
 * The array is in play only when the slices are merged by the separate merge
 * kernel (n_splits 1 or > 16, no schedulable cluster, ARCLLM_ATTN_CLUSTER=0);
 * the clustered form merges in distributed shared memory instead.
 * The first call on a device looks up the array's address (cudaGetSymbolAddress),
 * so make it outside stream capture. */
ARCLLM_CUDA_API int arcllm_cuda_attention_decode_noalloc(const float *q, const uint16_t *k_cache,
                                                         const uint16_t *v_cache, const uint32_t *pos_dev,
                                                         uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
                                                         uint32_t max_ctx, uint32_t layer, uint32_t n_splits,
                                                         float *out, void *stream);
/* Embedding row *token_dev of an F16 (1) or Q4_K (12) table into out[hidden]
 * (shaders/p8c_embedding_q4k_segmented_probe.comp, runtime.cpp:373). */
ARCLLM_CUDA_API int arcllm_cuda_embed(int type, const void *table, const uint32_t *token_dev, uint32_t hidden,
                                      uint32_t vocab, float *out, void *stream);
/* Greedy select over logits[n] (runtime_top2 top-1, runtime.cpp:132-148):
 * writes the first index of the maximum finite logit to *index_host and 1/0
 * to *finite_host (0 when any logit is non-finite).  Synchronous;
 * `scratch_dev` holds 16 bytes. */
ARCLLM_CUDA_API int arcllm_cuda_argmax(const float *logits, uint32_t n, void *scratch_dev, uint32_t *index_host,
                                       int *finite_host, void *stream);

/* ---- device memory and streams (for hosts that do not link the CUDA runtime) --- */
/* Launch overlap for the calling thread (programmatic dependent launch, as the
 * model's decode graphs use): while on, each kernel this thread launches may be
 * scheduled while its predecessor on the stream drains, streams its weights
 * before waiting for it, and waits for it before reading x, gamma, bias or
 * residual or writing its outputs.  Only for launch sequences whose weights no
 * preceding launch writes (e.g. back-to-back matvecs over constant weights,
 * captured in a CUDA graph).  Off by default; ARCLLM_PDL=0 disables it. */
ARCLLM_CUDA_API int arcllm_cuda_set_launch_overlap(int on);
ARCLLM_CUDA_API int arcllm_cuda_set_device(int device);
/* Number of visible CUDA devices (0 when none); fails only on a driver error. */
ARCLLM_CUDA_API int arcllm_cuda_device_count(int *out);
ARCLLM_CUDA_API int arcllm_cuda_malloc(uint64_t bytes, void **out);
ARCLLM_CUDA_API int arcllm_cuda_free(void *p);
ARCLLM_CUDA_API int arcllm_cuda_memcpy_h2d(void *dst, const void *src_host, uint64_t bytes, void *stream);
ARCLLM_CUDA_API int arcllm_cuda_memcpy_d2h(void *dst_host, const void *src, uint64_t bytes, void *stream);
ARCLLM_CUDA_API int arcllm_cuda_stream_create(void **out);
ARCLLM_CUDA_API int arcllm_cuda_stream_destroy(void *stream);
ARCLLM_CUDA_API int arcllm_cuda_stream_synchronize(void *stream);
/* Enqueues a one-thread kernel on `stream` that waits `us` microseconds of
 * device wall-clock time (%globaltimer), at most 1 s; used to start several
 * GPUs' timed work together after a device rendezvous. */
ARCLLM_CUDA_API int arcllm_cuda_stream_delay_us(uint32_t us, void *stream);

/* ---- greedy decode of one Qwen2-family model -----------------------------
 * The device half of arcllm::v1::runtime::generate() (src/arcllm_v1_runtime.cpp:
 * 149-536).  The caller owns the weight memory (device pointers into its
 * arenas); the model owns activations, an fp16 KV cache [layer][max_ctx]
 * [kv_heads*head_dim] (request-scoped, like the reference's :261-263), the
 * RoPE table and the device-side greedy state.  Each token is one CUDA-graph
 * launch; the next token is chosen on the device.  Not thread-safe per model. */
typedef struct arcllm_cuda_model arcllm_cuda_model;

typedef struct {
    uint32_t n_layers, hidden, n_heads, n_kv_heads, head_dim, ffn, vocab, max_ctx;
    float rms_eps;    /* GGUF qwen2.attention.layer_norm_rms_epsilon (runtime.cpp:183-184) */
    float rope_theta; /* GGUF qwen2.rope.freq_base (runtime.cpp:185-186) */
} arcllm_cuda_model_config;

/* One decoder block (tensor names of runtime.cpp:190-197).  Norms and biases
 * are fp32 device pointers; the type_* fields are ggml type ids. */
typedef struct {
    const float *attn_norm;
    const void *wq; const float *bq; int type_q;
    const void *wk; const float *bk; int type_k;
    const void *wv; const float *bv; int type_v;
    const void *wo; int type_o;
    const float *ffn_norm;
    const void *w_gate; const void *w_up; int type_gate_up;
    const void *w_down; int type_down;
} arcllm_cuda_layer;

/* Counters mirrored into arcllm::v1::runtime::RuntimeStats (runtime.h:25-46):
 * launches = kernel launches, graph launches = submits. */
typedef struct {
    uint32_t prefill_launches, prefill_graph_launches;
    uint32_t decode_launches_per_step, decode_graph_launches_per_step, decode_steps;
    float prefill_ms, decode_ms;
    int finite;
} arcllm_cuda_gen_stats;

ARCLLM_CUDA_API int arcllm_cuda_model_create(const arcllm_cuda_model_config *cfg, arcllm_cuda_model **out);
ARCLLM_CUDA_API int arcllm_cuda_model_destroy(arcllm_cuda_model *m);
ARCLLM_CUDA_API int arcllm_cuda_model_set_layer(arcllm_cuda_model *m, uint32_t layer, const arcllm_cuda_layer *w);
/* tok_embd_type: F16 (1, [vocab][hidden] halves) or Q4_K (12); output_type Q4_K/Q6_K */
ARCLLM_CUDA_API int arcllm_cuda_model_set_endpoints(arcllm_cuda_model *m, const void *tok_embd, int tok_embd_type,
                                                    const float *output_norm, const void *output, int output_type);
/* Greedy generation: consumes the prompt, then produces max_new tokens into
 * out_tokens_host.  Synchronous on `stream`.  Fails with ARC_E_NONFINITE on
 * non-finite logits (runtime.cpp:446,501).  In prefill mode 1 (the default)
 * all prompt tokens but the last go through the layers in batches of up to
 * 256 rows on the tcgen05 GEMMs (bf16 operands, fp32 accumulation; the
 * reference's prefill chain, runtime.cpp:340-369); in mode 0 (or with the
 * environment variable ARCLLM_PREFILL=token) one fp32 step per token. */
ARCLLM_CUDA_API int arcllm_cuda_model_generate(arcllm_cuda_model *m, const uint32_t *prompt_host, uint32_t n_prompt,
                                               uint32_t max_new, uint32_t *out_tokens_host,
                                               arcllm_cuda_gen_stats *stats, void *stream);
/* Step-level control (tests, benchmarks): begin() uploads the prompt and resets
 * the device state; step() enqueues one token step (with_head: output norm +
 * LM head + argmax) eagerly or as the captured graph. */
ARCLLM_CUDA_API int arcllm_cuda_model_begin(arcllm_cuda_model *m, const uint32_t *prompt_host, uint32_t n_prompt,
                                            uint32_t max_new, void *stream);
ARCLLM_CUDA_API int arcllm_cuda_model_step(arcllm_cuda_model *m, int with_head, int use_graph, void *stream);
/* After begin(): consume prompt tokens 0 .. n-2 the way generate() does (the
 * batched tensor-core prefill in mode 1, fp32 steps in mode 0; the reference's
 * prefill submit, src/arcllm_v1_runtime.cpp:340-369,440-446), so that the next
 * step(with_head = 1) yields the first generated token.  Once per begin(). */
ARCLLM_CUDA_API int arcllm_cuda_model_prefill(arcllm_cuda_model *m, void *stream);
/* Prefill mode: 1 = batched on the tensor cores (default), 0 = token by token. */
ARCLLM_CUDA_API int arcllm_cuda_model_set_prefill_mode(arcllm_cuda_model *m, int mode);
/* Q4_K/Q6_K down weights of `layer` for the batched prefill, needed when the
 * layer's decode down projection is bound to an EXEC148 image (type 148):
 * the prefill GEMMs read the GGUF packing.  Without it such a model prefills
 * token by token. */
ARCLLM_CUDA_API int arcllm_cuda_model_set_prefill_down(arcllm_cuda_model *m, uint32_t layer, const void *w, int type);
/* Device pointers to the last logits [vocab] and to the K / V caches. */
ARCLLM_CUDA_API int arcllm_cuda_model_logits(arcllm_cuda_model *m, const float **out);
ARCLLM_CUDA_API int arcllm_cuda_model_kv_cache(arcllm_cuda_model *m, const uint16_t **k, const uint16_t **v);
/* Restrict the LM head to rows [row0, row0+rows) of the output matrix given
 * to set_endpoints (row sharding across GPUs; the other rows of the logits
 * must be filled by the caller, e.g. all-gather, before the argmax reads all
 * vocab rows). */
ARCLLM_CUDA_API int arcllm_cuda_model_shard_lm_head(arcllm_cuda_model *m, uint32_t row0, uint32_t rows);
/* Tensor-parallel decode over n_ranks GPUs, one process and one model per
 * GPU, every rank holding the whole set of weights (the reference decodes on
 * one device, src/arcllm_v1_runtime.cpp:371-421).  Each rank runs the
 * attention half of every layer in full (replicated), its shard of the FFN
 * gate/up rows, the same K window (its slice of s) of the FFN down projection
 * and its shard of the LM-head rows; the ranks all-reduce the down
 * projection's partial sums (+ residual) and exchange their greedy-argmax
 * records over NVLink peer stores (the exchange kernel of
 * arcllm_cuda_exchange_gather), so every rank holds the full hidden state and
 * the global greedy token, and all ranks produce the same tokens.  rank_bufs
 * as for arcllm_cuda_exchange_gather with max_words from
 * arcllm_cuda_model_tp_exchange_words.  Every rank must call generate() (or
 * the same begin/prefill/step sequence) with the same arguments.  The logits
 * buffer (arcllm_cuda_model_logits) then holds this rank's LM-head rows only.
 * n_ranks == 1 turns it off. */
ARCLLM_CUDA_API int arcllm_cuda_model_tp_exchange_words(const arcllm_cuda_model_config *cfg, uint32_t n_ranks,
                                                        uint32_t *out);
ARCLLM_CUDA_API int arcllm_cuda_model_set_tensor_parallel(arcllm_cuda_model *m, void *const *rank_bufs,
                                                          uint32_t n_ranks, uint32_t rank, uint32_t timeout_us);

#ifdef __cplusplus
}
#endif
#endif /* ARCLLM_CUDA_H */
