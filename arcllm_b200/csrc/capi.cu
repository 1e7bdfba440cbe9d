// extern "C" entry points of libarcllm_cuda.so (declared in include/arcllm_cuda.h).
// Each one validates its arguments, maps failures to a status code and never
// lets a C++ exception or a CUDA error escape the ABI.
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <cstdlib>

#include "arcllm_cuda_internal.h"
#include "common.cuh"
#include "decode_ops.h"
#include "prefill_ops.h"

namespace arc {

int dequant(int fmt, const void* w, uint64_t n_blocks, float* y, cudaStream_t stream);
int fill_blocks(int fmt, void* w, uint64_t block_begin, uint64_t n_blocks, uint64_t seed, cudaStream_t stream);
int fill_normal(bool f16, void* y, uint64_t begin, uint64_t n, uint64_t seed, float mu, float sigma,
                cudaStream_t stream);

namespace {
thread_local char g_msg[512] = "";
__device__ unsigned int g_dev_error = 0;
}

unsigned int* dev_error_word() {
    static std::atomic<unsigned int*> cache[64] = {};  // per device; concurrent first calls store the same value
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        void* p = nullptr;  // outside the cache: resolve every time
        return cudaGetSymbolAddress(&p, g_dev_error) == cudaSuccess ? static_cast<unsigned int*>(p) : nullptr;
    }
    unsigned int* slot = cache[dev].load(std::memory_order_acquire);
    if (!slot) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_dev_error) != cudaSuccess) return nullptr;
        slot = static_cast<unsigned int*>(p);
        cache[dev].store(slot, std::memory_order_release);
    }
    return slot;
}

namespace {
thread_local bool g_pdl = false;
bool pdl_allowed() {
    static const bool allowed = [] {
        const char* e = std::getenv("ARCLLM_PDL");
        return !(e && e[0] == '0');
    }();
    return allowed;
}
}  // namespace

bool pdl_enabled() { return g_pdl && pdl_allowed(); }
PdlScope::PdlScope(bool on) : prev_(g_pdl) { g_pdl = on; }
PdlScope::~PdlScope() { g_pdl = prev_; }

int set_error(int status, const char* msg) {
    std::snprintf(g_msg, sizeof g_msg, "%s", msg ? msg : "");
    return status;
}

int set_cuda_error(cudaError_t e, const char* where) {
    std::snprintf(g_msg, sizeof g_msg, "%s: %s (%s)", where ? where : "cuda", cudaGetErrorName(e),
                  cudaGetErrorString(e));
    return e == cudaErrorMemoryAllocation ? ARC_E_OUT_OF_MEMORY : ARC_E_CUDA;
}

}  // namespace arc

using arc::set_error;

#define ARC_GUARD_BEGIN try {
#define ARC_GUARD_END                                                       \
    }                                                                       \
    catch (...) {                                                           \
        return set_error(ARC_E_INVALID_ARGUMENT, "unexpected C++ exception"); \
    }

extern "C" {

int arcllm_cuda_abi_version(void) { return ARCLLM_CUDA_ABI_VERSION; }

const char* arcllm_cuda_status_string(int status) {
    switch (status) {
        case ARC_OK: return "ARC_OK";
        case ARC_E_INVALID_ARGUMENT: return "ARC_E_INVALID_ARGUMENT";
        case ARC_E_ALIGNMENT: return "ARC_E_ALIGNMENT";
        case ARC_E_UNSUPPORTED_SHAPE: return "ARC_E_UNSUPPORTED_SHAPE";
        case ARC_E_CUDA: return "ARC_E_CUDA";
        case ARC_E_OUT_OF_MEMORY: return "ARC_E_OUT_OF_MEMORY";
        case ARC_E_DEVICE_TIMEOUT: return "ARC_E_DEVICE_TIMEOUT";
        case ARC_E_NONFINITE: return "ARC_E_NONFINITE";
        case ARC_E_NCCL: return "ARC_E_NCCL";
        default: return "ARC_E_UNKNOWN";
    }
}

const char* arcllm_cuda_last_error_message(void) { return arc::g_msg; }

int arcllm_cuda_device_error(void* stream, uint32_t* out_bits) {
    ARC_GUARD_BEGIN
    cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return arc::set_cuda_error(e, "device_error sync");
    unsigned int bits = 0, zero = 0;
    e = cudaMemcpyFromSymbol(&bits, arc::g_dev_error, sizeof bits);
    if (e != cudaSuccess) return arc::set_cuda_error(e, "device_error read");
    if (bits) {
        e = cudaMemcpyToSymbol(arc::g_dev_error, &zero, sizeof zero);
        if (e != cudaSuccess) return arc::set_cuda_error(e, "device_error clear");
    }
    if (out_bits) *out_bits = bits;
    if (bits & arc::ARC_DEV_ERR_TIMEOUT) return set_error(ARC_E_DEVICE_TIMEOUT, "a device-side wait timed out");
    return ARC_OK;
    ARC_GUARD_END
}

int arcllm_cuda_dequant_q4k(const void* w, uint64_t n_blocks, float* y, void* stream) {
    ARC_GUARD_BEGIN
    return arc::dequant(12, w, n_blocks, y, static_cast<cudaStream_t>(stream));
    ARC_GUARD_END
}

int arcllm_cuda_dequant_q6k(const void* w, uint64_t n_blocks, float* y, void* stream) {
    ARC_GUARD_BEGIN
    return arc::dequant(14, w, n_blocks, y, static_cast<cudaStream_t>(stream));
    ARC_GUARD_END
}

int arcllm_cuda_matvec(int ggml_type, const void* w, uint32_t rows, uint32_t k, const float* x, const float* gamma,
                       float eps, const float* bias, const float* residual, float* y, void* stream) {
    ARC_GUARD_BEGIN
    return arc::matvec_any(ggml_type, false, w, nullptr, rows, k, x, gamma, eps, bias, residual, y,
                           static_cast<cudaStream_t>(stream));
    ARC_GUARD_END
}

int arcllm_cuda_matvec_hostio(int ggml_type, const void* w, uint32_t rows, uint32_t k, const float* x_host,
                              float* x_dev, float* y_dev, float* y_host, void* stream) {
    ARC_GUARD_BEGIN
    if (!x_host || !y_host || !x_dev || !y_dev) return set_error(ARC_E_INVALID_ARGUMENT, "matvec_hostio: null pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(x_dev, x_host, sizeof(float) * k, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return arc::set_cuda_error(e, "matvec_hostio h2d");
    // Pinned (page-locked, device-mapped) y_host: the kernel stores the rows straight into it over
    // the host link while it streams the weights, as the reference's shaders write their output to
    // host-visible mapped memory.  Pageable y_host: y_dev, then one device-to-host copy.
    cudaPointerAttributes at{};
    const bool mapped = cudaPointerGetAttributes(&at, y_host) == cudaSuccess && at.type == cudaMemoryTypeHost &&
                        at.devicePointer != nullptr;
    if (!mapped) cudaGetLastError();  // clear a lookup failure of an unregistered pointer
    float* y_out = mapped ? static_cast<float*>(at.devicePointer) : y_dev;
    int st = arc::matvec_any(ggml_type, false, w, nullptr, rows, k, x_dev, nullptr, 0.f, nullptr, nullptr, y_out, s);
    if (st != ARC_OK) return st;
    if (!mapped) {
        e = cudaMemcpyAsync(y_host, y_dev, sizeof(float) * rows, cudaMemcpyDeviceToHost, s);
        if (e != cudaSuccess) return arc::set_cuda_error(e, "matvec_hostio d2h");
    }
    e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return arc::set_cuda_error(e, "matvec_hostio sync");
    return ARC_OK;
    ARC_GUARD_END
}

// ---- rank all-gather over NVLink peer memory ----
// Exchange buffer of one rank: the word array [rows_total] of 64-bit (epoch << 32 | fp32 bits)
// words at 0, which every rank's launch stores into, then at a 256-byte boundary the fp32
// logits [rows_total] this rank's own launches collect from it.
static uint64_t gather_logits_offset(uint32_t rows_total) {
    return ((uint64_t)rows_total * 8u + 255u) & ~uint64_t(255);
}

int arcllm_cuda_allgather_buffer_bytes(uint32_t rows_total, uint64_t* out) {
    ARC_GUARD_BEGIN
    if (!out || rows_total == 0) return set_error(ARC_E_INVALID_ARGUMENT, "allgather_buffer_bytes: bad argument");
    *out = gather_logits_offset(rows_total) + (((uint64_t)rows_total * 4u + 255u) & ~uint64_t(255));
    return ARC_OK;
    ARC_GUARD_END
}

int arcllm_cuda_allgather_logits_offset(uint32_t rows_total, uint64_t* out) {
    ARC_GUARD_BEGIN
    if (!out || rows_total == 0) return set_error(ARC_E_INVALID_ARGUMENT, "allgather_logits_offset: bad argument");
    *out = gather_logits_offset(rows_total);
    return ARC_OK;
    ARC_GUARD_END
}

// Checks the arguments of one all-gather matvec and fills its RankGather (g.out = this rank's logits
// in its own exchange buffer).  Shared by the device-resident and the host-IO entry points.
static int allgather_setup(int ggml_type, uint32_t rows, uint32_t k, const float* x, uint32_t row0,
                           uint32_t rows_total, void* const* rank_bufs, uint32_t n_ranks, uint32_t rank,
                           uint32_t epoch, uint32_t timeout_us, arc::RankGather& g) {
    if (ggml_type != ARC_GGML_Q4_K && ggml_type != ARC_GGML_Q6_K)
        return set_error(ARC_E_INVALID_ARGUMENT, "matvec_allgather: Q4_K or Q6_K weights");
    if (!rank_bufs || n_ranks == 0 || n_ranks > 8 || rank >= n_ranks || epoch == 0 || rows == 0 ||
        (uint64_t)row0 + rows > rows_total)
        return set_error(ARC_E_INVALID_ARGUMENT, "matvec_allgather: bad rank layout or epoch");
    if (!arc::matvec_imma_supported(ggml_type, false, rows, k) || (reinterpret_cast<uintptr_t>(x) & 15u))
        return set_error(ARC_E_UNSUPPORTED_SHAPE, "matvec_allgather: needs the whole-row tensor-core kernel "
                                                  "(K/256 <= 14, 16-byte aligned x)");
    g = arc::RankGather{};
    g.n_ranks = n_ranks;
    g.self_rank = rank;
    g.epoch = epoch;
    g.row0 = row0;
    g.rows_total = rows_total;
    g.wait_ns = 1000ull * (timeout_us ? timeout_us : 2000000u);
    for (uint32_t r = 0; r < n_ranks; ++r) {
        if (!rank_bufs[r] || (reinterpret_cast<uintptr_t>(rank_bufs[r]) & 255u))
            return set_error(ARC_E_ALIGNMENT, "matvec_allgather: rank buffers must be 256-byte aligned");
        g.ll[r] = static_cast<unsigned long long*>(rank_bufs[r]);
    }
    g.out = reinterpret_cast<float*>(static_cast<uint8_t*>(rank_bufs[rank]) + gather_logits_offset(rows_total));
    return ARC_OK;
}

int arcllm_cuda_matvec_allgather(int ggml_type, const void* w, uint32_t rows, uint32_t k, const float* x,
                                 uint32_t row0, uint32_t rows_total, void* const* rank_bufs, uint32_t n_ranks,
                                 uint32_t rank, uint32_t epoch, uint32_t timeout_us, void* stream) {
    ARC_GUARD_BEGIN
    arc::RankGather g;
    const int st = allgather_setup(ggml_type, rows, k, x, row0, rows_total, rank_bufs, n_ranks, rank, epoch,
                                   timeout_us, g);
    if (st != ARC_OK) return st;
    return arc::matvec_imma_launch(ggml_type, false, w, nullptr, rows, k, x, nullptr, 0.f, nullptr, nullptr,
                                   g.out + row0, static_cast<cudaStream_t>(stream), nullptr, &g);
    ARC_GUARD_END
}

int arcllm_cuda_matvec_allgather_hostio(int ggml_type, const void* w, uint32_t rows, uint32_t k,
                                        const float* x_host, float* x_dev, uint32_t row0, uint32_t rows_total,
                                        void* const* rank_bufs, uint32_t n_ranks, uint32_t rank, uint32_t epoch,
                                        uint32_t timeout_us, float* y_host, void* stream) {
    ARC_GUARD_BEGIN
    if (!x_host || !y_host || !x_dev) return set_error(ARC_E_INVALID_ARGUMENT, "matvec_allgather_hostio: null pointer");
    arc::RankGather g;
    int st = allgather_setup(ggml_type, rows, k, x_dev, row0, rows_total, rank_bufs, n_ranks, rank, epoch,
                             timeout_us, g);
    if (st != ARC_OK) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(x_dev, x_host, sizeof(float) * k, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return arc::set_cuda_error(e, "matvec_allgather_hostio h2d");
    // Pinned, device-mapped y_host: the collect phase stores every rank's rows straight into it, so
    // each logit crosses the host link once and no copy follows the kernel (this rank's own rows still
    // go to its device buffer, which nothing reads).  Pageable y_host: the device logits, then one copy.
    cudaPointerAttributes at{};
    const bool mapped = cudaPointerGetAttributes(&at, y_host) == cudaSuccess && at.type == cudaMemoryTypeHost &&
                        at.devicePointer != nullptr;
    if (!mapped) cudaGetLastError();  // clear a lookup failure of an unregistered pointer
    float* const own = g.out;
    if (mapped) g.out = static_cast<float*>(at.devicePointer);
    st = arc::matvec_imma_launch(ggml_type, false, w, nullptr, rows, k, x_dev, nullptr, 0.f, nullptr, nullptr,
                                 own + row0, s, nullptr, &g);
    if (st != ARC_OK) return st;
    if (!mapped) {
        e = cudaMemcpyAsync(y_host, own, sizeof(float) * rows_total, cudaMemcpyDeviceToHost, s);
        if (e != cudaSuccess) return arc::set_cuda_error(e, "matvec_allgather_hostio d2h");
    }
    e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return arc::set_cuda_error(e, "matvec_allgather_hostio sync");
    return ARC_OK;
    ARC_GUARD_END
}

int arcllm_cuda_ipc_get_handle(const void* dev_ptr, void* handle_out) {
    ARC_GUARD_BEGIN
    if (!dev_ptr || !handle_out) return set_error(ARC_E_INVALID_ARGUMENT, "ipc_get_handle: null pointer");
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr));
    if (e != cudaSuccess) return arc::set_cuda_error(e, "ipc_get_handle");
    std::memcpy(handle_out, &h, sizeof(h));
    return ARC_OK;
    ARC_GUARD_END
}

int arcllm_cuda_ipc_open_handle(const void* handle, void** dev_ptr_out) {
    ARC_GUARD_BEGIN
    if (!handle || !dev_ptr_out) return set_error(ARC_E_INVALID_ARGUMENT, "ipc_open_handle: null pointer");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    cudaError_t e = cudaIpcOpenMemHandle(dev_ptr_out, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return arc::set_cuda_error(e, "ipc_open_handle");
    return ARC_OK;
    ARC_GUARD_END
}

int arcllm_cuda_ipc_close_handle(void* dev_ptr) {
    ARC_GUARD_BEGIN
    if (!dev_ptr) return set_error(ARC_E_INVALID_ARGUMENT, "ipc_close_handle: null pointer");
    cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
    if (e != cudaSuccess) return arc::set_cuda_error(e, "ipc_close_handle");
    return ARC_OK;
    ARC_GUARD_END
}

int arcllm_cuda_exchange_buffer_bytes(uint32_t max_words, uint64_t* out) {
    ARC_GUARD_BEGIN
    if (!out || max_words == 0) return set_error(ARC_E_INVALID_ARGUMENT, "exchange_buffer_bytes: bad argument");
    *out = arc::exchange_buffer_bytes(max_words);
    return ARC_OK;
    ARC_GUARD_END
}

int arcllm_cuda_exchange_gather(void* const* rank_bufs, uint32_t n_ranks, uint32_t rank, uint32_t max_words,
                                const void* src, uint32_t n_local, uint32_t offset, void* dst, uint32_t n_total,
                                uint32_t timeout_us, void* stream) {
    ARC_GUARD_BEGIN
    if (!rank_bufs || n_ranks == 0 || n_ranks > 8 || rank >= n_ranks)
        return set_error(ARC_E_INVALID_ARGUMENT, "exchange_gather: 1..8 ranks, rank < n_ranks");
    arc::ExchangeRanks ex{};
    for (uint32_t q = 0; q < n_ranks; ++q) ex.bufs[q] = rank_bufs[q];
    ex.n_ranks = n_ranks;
    ex.rank = rank;
    ex.max_words = max_words;
    ex.timeout_us = timeout_us;
    return arc::exchange_gather(ex, src, n_local, offset, dst, n_total, static_cast<cudaStream_t>(stream));
    ARC_GUARD_END
}

int arcllm_cuda_shard_rows(uint32_t n, uint32_t align, uint32_t n_ranks, uint32_t rank, uint32_t* row0,
                           uint32_t* rows) {
    ARC_GUARD_BEGIN
    return arc::shard_rows(n, align, n_ranks, rank, row0, rows);
    ARC_GUARD_END
}

int arcllm_cuda_matvec_q4k(const void* w, uint32_t rows, uint32_t k, const float* x, const float* bias, float* y,
                           void* stream) {
    return arcllm_cuda_matvec(ARC_GGML_Q4_K, w, rows, k, x, nullptr, 0.f, bias, nullptr, y, stream);
}

int arcllm_cuda_matvec_q6k(const void* w, uint32_t rows, uint32_t k, const float* x, const float* bias, float* y,
                           void* stream) {
    return arcllm_cuda_matvec(ARC_GGML_Q6_K, w, rows, k, x, nullptr, 0.f, bias, nullptr, y, stream);
}

int arcllm_cuda_gateup_silu_q4k(const void* w_gate, const void* w_up, uint32_t rows, uint32_t k, const float* x,
                                const float* gamma, float eps, float* s, void* stream) {
    ARC_GUARD_BEGIN
    return arc::matvec_any(ARC_GGML_Q4_K, true, w_gate, w_up, rows, k, x, gamma, eps, nullptr, nullptr, s,
                           static_cast<cudaStream_t>(stream));
    ARC_GUARD_END
}

int arcllm_cuda_ffn_block(int down_type, const void* w_gate, const void* w_up, const void* w_down, uint32_t hidden,
                          uint32_t ffn, const float* x, const float* gamma, float eps, float* s,
                          const float* residual, float* y, void* stream) {
    ARC_GUARD_BEGIN
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    int rc = arc::matvec_any(ARC_GGML_Q4_K, true, w_gate, w_up, ffn, hidden, x, gamma, eps, nullptr, nullptr, s, st);
    if (rc == ARC_OK)
        rc = arc::matvec_any(down_type, false, w_down, nullptr, hidden, ffn, s, nullptr, 0.f, nullptr, residual, y, st);
    return rc;
    ARC_GUARD_END
}

int arcllm_cuda_exec148_materialize(const void* q4k, uint64_t n_blocks, void* exec, void* stream) {
    ARC_GUARD_BEGIN
    return arc::exec148_materialize(q4k, n_blocks, exec, static_cast<cudaStream_t>(stream));
    ARC_GUARD_END
}

int arcllm_cuda_exec148_validate(const void* q4k, const void* exec, uint64_t n_blocks, uint64_t* mismatches_host,
                                 void* stream) {
    ARC_GUARD_BEGIN
    return arc::exec148_validate(q4k, exec, n_blocks, mismatches_host, static_cast<cudaStream_t>(stream));
    ARC_GUARD_END
}

int arcllm_cuda_gemm_q4k_bf16(const void* w, uint32_t n, uint32_t k, const uint16_t* x_bf16, uint32_t m, float* y,
                              void* stream) {
    ARC_GUARD_BEGIN
    return arc::gemm_q4k_bf16(w, n, k, x_bf16, m, y, static_cast<cudaStream_t>(stream));
    ARC_GUARD_END
}

int arcllm_cuda_gemm_allgather_buffer_bytes(uint32_t m, uint32_t n_total, uint64_t* out) {
    ARC_GUARD_BEGIN
    if (!out || m == 0 || n_total == 0)
        return set_error(ARC_E_INVALID_ARGUMENT, "gemm_allgather_buffer_bytes: bad argument");
    *out = arc::gemm_gather_flags_offset(m, n_total) + 128u;
    return ARC_OK;
    ARC_GUARD_END
}

int arcllm_cuda_gemm_bf16_allgather(int type, const void* w, uint32_t n, uint32_t k, const uint16_t* x_bf16,
                                    uint32_t m, uint32_t c0, uint32_t n_total, void* const* rank_bufs,
                                    uint32_t n_ranks, uint32_t rank, uint32_t epoch, uint32_t timeout_us,
                                    void* stream) {
    ARC_GUARD_BEGIN
    return arc::gemm_kq_allgather(type, w, n, k, x_bf16, m, c0, n_total, rank_bufs, n_ranks, rank, epoch, timeout_us,
                                  static_cast<cudaStream_t>(stream));
    ARC_GUARD_END
}

int arcllm_cuda_gemm_bf16(int type, const void* w, uint32_t n, uint32_t k, const uint16_t* x_bf16, uint32_t m,
                          const float* residual, float* y, void* stream) {
    ARC_GUARD_BEGIN
    return arc::gemm_kq_bf16(type, w, n, k, x_bf16, m, residual, y, static_cast<cudaStream_t>(stream));
    ARC_GUARD_END
}

int arcllm_cuda_gemm_f16(int type, const void* w, uint32_t n, uint32_t k, const uint16_t* x_f16, uint32_t m,
                         const float* residual, float* y, void* stream) {
    ARC_GUARD_BEGIN
    return arc::gemm_kq_bf16(type, w, n, k, x_f16, m, residual, y, static_cast<cudaStream_t>(stream), 1);
    ARC_GUARD_END
}

int arcllm_cuda_gemm_f16x3(int type, const void* w, uint32_t n, uint32_t k, const uint16_t* x_hi,
                           const uint16_t* x_lo, uint32_t m, const float* residual, float* y, void* stream) {
    ARC_GUARD_BEGIN
    if (!x_lo) return arc::set_error(ARC_E_INVALID_ARGUMENT, "gemm f16x3: null x_lo");
    return arc::gemm_kq_bf16(type, w, n, k, x_hi, m, residual, y, static_cast<cudaStream_t>(stream), 2, x_lo);
    ARC_GUARD_END
}

int arcllm_cuda_rmsnorm_rows(const float* x, const float* gamma, float eps, uint32_t rows, uint32_t h, int out_fp16,
                             uint16_t* out, uint16_t* out_lo, void* stream) {
    ARC_GUARD_BEGIN
    if (out_lo && !out_fp16) return arc::set_error(ARC_E_INVALID_ARGUMENT, "rmsnorm rows: out_lo needs fp16 output");
    return arc::launch_rmsnorm_rows_bf16(x, gamma, eps, rows, h, out, static_cast<cudaStream_t>(stream),
                                         out_fp16 != 0, out_lo);
    ARC_GUARD_END
}

int arcllm_cuda_fill_q4k(void* w, uint64_t block_begin, uint64_t n_blocks, uint64_t seed, void* stream) {
    ARC_GUARD_BEGIN
    return arc::fill_blocks(12, w, block_begin, n_blocks, seed, static_cast<cudaStream_t>(stream));
    ARC_GUARD_END
}

int arcllm_cuda_fill_q6k(void* w, uint64_t block_begin, uint64_t n_blocks, uint64_t seed, void* stream) {
    ARC_GUARD_BEGIN
    return arc::fill_blocks(14, w, block_begin, n_blocks, seed, static_cast<cudaStream_t>(stream));
    ARC_GUARD_END
}

int arcllm_cuda_fill_normal_f32(float* y, uint64_t begin, uint64_t n, uint64_t seed, float mu, float sigma,
                                void* stream) {
    ARC_GUARD_BEGIN
    return arc::fill_normal(false, y, begin, n, seed, mu, sigma, static_cast<cudaStream_t>(stream));
    ARC_GUARD_END
}

int arcllm_cuda_fill_normal_f16(uint16_t* y, uint64_t begin, uint64_t n, uint64_t seed, float mu, float sigma,
                                void* stream) {
    ARC_GUARD_BEGIN
    return arc::fill_normal(true, y, begin, n, seed, mu, sigma, static_cast<cudaStream_t>(stream));
    ARC_GUARD_END
}

int arcllm_cuda_rope_table(float* table, uint32_t max_ctx, uint32_t head_dim, float theta) {
    ARC_GUARD_BEGIN
    if (!table || max_ctx == 0 || head_dim == 0 || (head_dim & 1u))
        return set_error(ARC_E_INVALID_ARGUMENT, "rope_table: bad arguments");
    std::vector<float> t = arc::rope_table(max_ctx, head_dim, theta);
    const cudaError_t e = cudaMemcpy(table, t.data(), t.size() * sizeof(float), cudaMemcpyHostToDevice);
    return e == cudaSuccess ? ARC_OK : arc::set_cuda_error(e, "rope_table");
    ARC_GUARD_END
}

int arcllm_cuda_rope_kv_store(float* q, float* k, const float* v, const float* table, const uint32_t* pos_dev,
                              uint16_t* k_cache, uint16_t* v_cache, uint32_t q_heads, uint32_t kv_heads,
                              uint32_t head_dim, uint32_t max_ctx, uint32_t layer, void* stream) {
    ARC_GUARD_BEGIN
    if (!q || !k || !v || !table || !pos_dev || !k_cache || !v_cache)
        return set_error(ARC_E_INVALID_ARGUMENT, "rope_kv_store: null pointer");
    if (head_dim == 0 || (head_dim & 1u) || q_heads == 0 || kv_heads == 0 || max_ctx == 0)
        return set_error(ARC_E_INVALID_ARGUMENT, "rope_kv_store: bad shape");
    arc::RopeKvShape s{q_heads, kv_heads, head_dim, max_ctx, layer};
    return arc::launch_rope_kv_store(q, k, v, reinterpret_cast<const float2*>(table), pos_dev, k_cache, v_cache, s,
                                     static_cast<cudaStream_t>(stream));
    ARC_GUARD_END
}

int arcllm_cuda_attention_decode(const float* q, const uint16_t* k_cache, const uint16_t* v_cache,
                                 const uint32_t* pos_dev, uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
                                 uint32_t max_ctx, uint32_t layer, uint32_t n_splits, float* scratch, float* out,
                                 void* stream) {
    ARC_GUARD_BEGIN
    if (!q || !k_cache || !v_cache || !pos_dev || !scratch || !out)
        return set_error(ARC_E_INVALID_ARGUMENT, "attention: null pointer");
    if (n_splits == 0 || n_splits > 65535u || kv_heads == 0 || max_ctx == 0)
        return set_error(ARC_E_INVALID_ARGUMENT, "attention: bad shape");
    arc::AttnShape s{q_heads, kv_heads, head_dim, max_ctx, layer, n_splits, 1.0f / std::sqrt((float)head_dim)};
    return arc::launch_attention(q, k_cache, v_cache, pos_dev, s, scratch, out, static_cast<cudaStream_t>(stream));
    ARC_GUARD_END
}

int arcllm_cuda_rope_kv_rows(float* q, float* k, const float* v, const float* bq, const float* bk, const float* bv,
                             const float* table, uint32_t pos0, uint32_t rows, uint16_t* k_cache, uint16_t* v_cache,
                             uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim, uint32_t max_ctx, uint32_t layer,
                             void* stream) {
    ARC_GUARD_BEGIN
    if (!q || !k || !v || !table || !k_cache || !v_cache) return set_error(ARC_E_INVALID_ARGUMENT, "rope rows: null");
    if (head_dim == 0 || head_dim % 2u || kv_heads == 0 || q_heads == 0 || max_ctx == 0)
        return set_error(ARC_E_INVALID_ARGUMENT, "rope rows: bad shape");
    arc::RopeKvShape s{q_heads, kv_heads, head_dim, max_ctx, layer};
    return arc::launch_rope_kv_rows(q, k, v, bq, bk, bv, reinterpret_cast<const float2*>(table), pos0, rows, k_cache,
                                    v_cache, s, static_cast<cudaStream_t>(stream));
    ARC_GUARD_END
}

int arcllm_cuda_attention_prefill(const float* q, const uint16_t* k_cache, const uint16_t* v_cache, uint32_t pos0,
                                  uint32_t rows, uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
                                  uint32_t max_ctx, uint32_t layer, uint16_t* out_bf16, void* stream) {
    ARC_GUARD_BEGIN
    if (!q || !k_cache || !v_cache || !out_bf16) return set_error(ARC_E_INVALID_ARGUMENT, "attention prefill: null");
    if (kv_heads == 0 || max_ctx == 0 || rows > 65535u) return set_error(ARC_E_INVALID_ARGUMENT, "attention prefill: bad shape");
    arc::AttnShape s{q_heads, kv_heads, head_dim, max_ctx, layer, 1, 1.0f / std::sqrt((float)head_dim)};
    return arc::launch_attention_prefill(q, k_cache, v_cache, pos0, rows, s, out_bf16, static_cast<cudaStream_t>(stream));
    ARC_GUARD_END
}

int arcllm_cuda_embed(int type, const void* table, const uint32_t* token_dev, uint32_t hidden, uint32_t vocab,
                      float* out, void* stream) {
    ARC_GUARD_BEGIN
    if (!table || !token_dev || !out || hidden == 0) return set_error(ARC_E_INVALID_ARGUMENT, "embed: bad arguments");
    if (type == ARC_GGML_Q4_K && (hidden % 256u)) return set_error(ARC_E_INVALID_ARGUMENT, "embed: Q4_K rows need hidden % 256 == 0");
    return arc::launch_embed(type, table, token_dev, hidden, vocab, out, static_cast<cudaStream_t>(stream));
    ARC_GUARD_END
}

int arcllm_cuda_argmax(const float* logits, uint32_t n, void* scratch_dev, uint32_t* index_host, int* finite_host,
                       void* stream) {
    ARC_GUARD_BEGIN
    if (!logits || !scratch_dev || !index_host || n == 0)
        return set_error(ARC_E_INVALID_ARGUMENT, "argmax: bad arguments");
    if (reinterpret_cast<uintptr_t>(scratch_dev) & 7u) return set_error(ARC_E_ALIGNMENT, "argmax: scratch 8-byte alignment");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    unsigned long long* key = static_cast<unsigned long long*>(scratch_dev);
    uint32_t* flag = reinterpret_cast<uint32_t*>(key + 1);
    cudaError_t e = cudaMemsetAsync(scratch_dev, 0, 16, s);
    if (e != cudaSuccess) return arc::set_cuda_error(e, "argmax clear");
    int st = arc::launch_argmax(logits, n, key, flag, s);
    if (st != ARC_OK) return st;
    unsigned long long hk[2] = {0, 0};
    e = cudaMemcpyAsync(hk, scratch_dev, 16, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return arc::set_cuda_error(e, "argmax read");
    const uint32_t nonfinite = (uint32_t)(hk[1] & 0xffffffffull);
    *index_host = hk[0] ? ~(uint32_t)(hk[0] & 0xffffffffull) : 0u;
    if (finite_host) *finite_host = (nonfinite == 0 && hk[0] != 0) ? 1 : 0;
    return ARC_OK;
    ARC_GUARD_END
}

int arcllm_cuda_set_launch_overlap(int on) {
    ARC_GUARD_BEGIN
    arc::g_pdl = on != 0;
    return ARC_OK;
    ARC_GUARD_END
}

int arcllm_cuda_set_device(int device) {
    const cudaError_t e = cudaSetDevice(device);
    return e == cudaSuccess ? ARC_OK : arc::set_cuda_error(e, "set_device");
}

int arcllm_cuda_device_count(int* out) {
    if (!out) return set_error(ARC_E_INVALID_ARGUMENT, "device_count: null out");
    *out = 0;
    const cudaError_t e = cudaGetDeviceCount(out);
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) {
        cudaGetLastError();
        *out = 0;
        return ARC_OK;
    }
    return e == cudaSuccess ? ARC_OK : arc::set_cuda_error(e, "device_count");
}

int arcllm_cuda_malloc(uint64_t bytes, void** out) {
    if (!out) return set_error(ARC_E_INVALID_ARGUMENT, "malloc: null out");
    const cudaError_t e = cudaMalloc(out, bytes);
    return e == cudaSuccess ? ARC_OK : arc::set_cuda_error(e, "malloc");
}

int arcllm_cuda_free(void* p) {
    const cudaError_t e = cudaFree(p);
    return e == cudaSuccess ? ARC_OK : arc::set_cuda_error(e, "free");
}

int arcllm_cuda_memcpy_h2d(void* dst, const void* src_host, uint64_t bytes, void* stream) {
    const cudaError_t e = cudaMemcpyAsync(dst, src_host, bytes, cudaMemcpyHostToDevice, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? ARC_OK : arc::set_cuda_error(e, "memcpy_h2d");
}

int arcllm_cuda_memcpy_d2h(void* dst_host, const void* src, uint64_t bytes, void* stream) {
    const cudaError_t e = cudaMemcpyAsync(dst_host, src, bytes, cudaMemcpyDeviceToHost, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? ARC_OK : arc::set_cuda_error(e, "memcpy_d2h");
}

int arcllm_cuda_stream_create(void** out) {
    if (!out) return set_error(ARC_E_INVALID_ARGUMENT, "stream_create: null out");
    cudaStream_t s;
    const cudaError_t e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
    if (e != cudaSuccess) return arc::set_cuda_error(e, "stream_create");
    *out = s;
    return ARC_OK;
}

int arcllm_cuda_stream_destroy(void* stream) {
    const cudaError_t e = cudaStreamDestroy(static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? ARC_OK : arc::set_cuda_error(e, "stream_destroy");
}

int arcllm_cuda_stream_synchronize(void* stream) {
    const cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? ARC_OK : arc::set_cuda_error(e, "stream_synchronize");
}

namespace {
// One thread polls %globaltimer until `ns` nanoseconds have passed: the same wall-clock delay on every
// GPU whatever its SM clock (a cycle-count spin ends up to ~10 % apart between GPUs at different clocks).
__global__ void stream_delay_kernel(unsigned long long ns) {
    const unsigned long long t0 = arc::globaltimer();
    while (arc::globaltimer() - t0 < ns) __nanosleep(1000);
}
}  // namespace

int arcllm_cuda_stream_delay_us(uint32_t us, void* stream) {
    if (us > 1000000u) return set_error(ARC_E_INVALID_ARGUMENT, "stream_delay_us: at most 1 s");
    stream_delay_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(1000ull * us);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ARC_OK : arc::set_cuda_error(e, "stream_delay_us");
}

int arcllm_cuda_model_create(const arcllm_cuda_model_config* cfg, arcllm_cuda_model** out) {
    ARC_GUARD_BEGIN
    return arc::model_create(cfg, out);
    ARC_GUARD_END
}

int arcllm_cuda_model_destroy(arcllm_cuda_model* m) {
    ARC_GUARD_BEGIN
    return arc::model_destroy(m);
    ARC_GUARD_END
}

int arcllm_cuda_model_set_layer(arcllm_cuda_model* m, uint32_t layer, const arcllm_cuda_layer* w) {
    ARC_GUARD_BEGIN
    return arc::model_set_layer(m, layer, w);
    ARC_GUARD_END
}

int arcllm_cuda_model_set_endpoints(arcllm_cuda_model* m, const void* tok_embd, int tok_embd_type,
                                    const float* output_norm, const void* output, int output_type) {
    ARC_GUARD_BEGIN
    return arc::model_set_endpoints(m, tok_embd, tok_embd_type, output_norm, output, output_type);
    ARC_GUARD_END
}

int arcllm_cuda_model_generate(arcllm_cuda_model* m, const uint32_t* prompt_host, uint32_t n_prompt, uint32_t max_new,
                               uint32_t* out_tokens_host, arcllm_cuda_gen_stats* stats, void* stream) {
    ARC_GUARD_BEGIN
    return arc::model_generate(m, prompt_host, n_prompt, max_new, out_tokens_host, stats,
                               static_cast<cudaStream_t>(stream));
    ARC_GUARD_END
}

int arcllm_cuda_model_begin(arcllm_cuda_model* m, const uint32_t* prompt_host, uint32_t n_prompt, uint32_t max_new,
                            void* stream) {
    ARC_GUARD_BEGIN
    return arc::model_begin(m, prompt_host, n_prompt, max_new, static_cast<cudaStream_t>(stream));
    ARC_GUARD_END
}

int arcllm_cuda_model_tp_exchange_words(const arcllm_cuda_model_config* cfg, uint32_t n_ranks, uint32_t* out) {
    ARC_GUARD_BEGIN
    return arc::model_tp_exchange_words(cfg, n_ranks, out);
    ARC_GUARD_END
}

int arcllm_cuda_model_set_tensor_parallel(arcllm_cuda_model* m, void* const* rank_bufs, uint32_t n_ranks,
                                          uint32_t rank, uint32_t timeout_us) {
    ARC_GUARD_BEGIN
    return arc::model_set_tensor_parallel(m, rank_bufs, n_ranks, rank, timeout_us);
    ARC_GUARD_END
}

int arcllm_cuda_model_prefill(arcllm_cuda_model* m, void* stream) {
    ARC_GUARD_BEGIN
    return arc::model_prefill(m, static_cast<cudaStream_t>(stream), nullptr);
    ARC_GUARD_END
}

int arcllm_cuda_model_step(arcllm_cuda_model* m, int with_head, int use_graph, void* stream) {
    ARC_GUARD_BEGIN
    return arc::model_step(m, with_head, use_graph, static_cast<cudaStream_t>(stream));
    ARC_GUARD_END
}

int arcllm_cuda_model_set_prefill_mode(arcllm_cuda_model* m, int mode) {
    ARC_GUARD_BEGIN
    return arc::model_set_prefill_mode(m, mode);
    ARC_GUARD_END
}

int arcllm_cuda_model_set_prefill_down(arcllm_cuda_model* m, uint32_t layer, const void* w, int type) {
    ARC_GUARD_BEGIN
    return arc::model_set_prefill_down(m, layer, w, type);
    ARC_GUARD_END
}

int arcllm_cuda_model_logits(arcllm_cuda_model* m, const float** out) {
    ARC_GUARD_BEGIN
    return arc::model_logits(m, out);
    ARC_GUARD_END
}

int arcllm_cuda_model_kv_cache(arcllm_cuda_model* m, const uint16_t** k, const uint16_t** v) {
    ARC_GUARD_BEGIN
    return arc::model_kv_cache(m, k, v);
    ARC_GUARD_END
}

int arcllm_cuda_model_shard_lm_head(arcllm_cuda_model* m, uint32_t row0, uint32_t rows) {
    ARC_GUARD_BEGIN
    return arc::model_shard_lm_head(m, row0, rows);
    ARC_GUARD_END
}

}  // extern "C"
