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

ARCLLM_CUDA_API int arcllm_cuda_abi_version(void);
ARCLLM_CUDA_API const char *arcllm_cuda_status_string(int status);
ARCLLM_CUDA_API const char *arcllm_cuda_last_error_message(void);

/* Reads (and clears) the device error word the kernels set when a bounded
 * wait gives up (bit 0) or an index check fails (bit 1).  Synchronises
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
 * x_dev, runs arcllm_cuda_matvec (no norm/bias/residual), copies rows floats
 * y_dev -> y_host and waits for `stream`.  x_dev / y_dev are caller-owned
 * device buffers; host buffers should be pinned for asynchronous copies. */
ARCLLM_CUDA_API int arcllm_cuda_matvec_hostio(int ggml_type, const void *w, uint32_t rows, uint32_t k,
                                              const float *x_host, float *x_dev, float *y_dev, float *y_host,
                                              void *stream);

/* ---- fused gate/up projection with SiLU-multiply (Q4_K) -------------------
 * s[r] = silu(g[r]) * u[r],  g = W_gate . xn,  u = W_up . xn,  xn as above.
 * Replaces the I002 pair of shaders/sa1_q4k_subgroup_splitk.comp dispatches
 * plus shaders/p7_swiglu.comp (src/arcllm_v1_runtime.cpp:390-405) and the
 * ffn_norm shaders/p7_rmsnorm_seq.comp before them (:389). */
ARCLLM_CUDA_API int arcllm_cuda_gateup_silu_q4k(const void *w_gate, const void *w_up, uint32_t rows, uint32_t k,
                                const float *x, const float *gamma, float eps, float *s, void *stream);

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

#ifdef __cplusplus
}
#endif
#endif /* ARCLLM_CUDA_H */
