// extern "C" entry points of libarcllm_cuda.so (declared in include/arcllm_cuda.h).
// Each one validates its arguments, maps failures to a status code and never
// lets a C++ exception or a CUDA error escape the ABI.
#include <cstdio>
#include <cstring>

#include "arcllm_cuda_internal.h"
#include "common.cuh"

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
    static unsigned int* cache[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    unsigned int*& slot = cache[dev & 63];
    if (!slot) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_dev_error) != cudaSuccess) return nullptr;
        slot = static_cast<unsigned int*>(p);
    }
    return slot;
}

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
    arc::MatvecPlan pl;
    int st = arc::matvec_plan(ggml_type, false, rows, k, &pl);
    if (st != ARC_OK) return st;
    return arc::matvec_launch(pl, w, nullptr, x, gamma, eps, bias, residual, y, static_cast<cudaStream_t>(stream));
    ARC_GUARD_END
}

int arcllm_cuda_matvec_hostio(int ggml_type, const void* w, uint32_t rows, uint32_t k, const float* x_host,
                              float* x_dev, float* y_dev, float* y_host, void* stream) {
    ARC_GUARD_BEGIN
    if (!x_host || !y_host || !x_dev || !y_dev) return set_error(ARC_E_INVALID_ARGUMENT, "matvec_hostio: null pointer");
    arc::MatvecPlan pl;
    int st = arc::matvec_plan(ggml_type, false, rows, k, &pl);
    if (st != ARC_OK) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(x_dev, x_host, sizeof(float) * k, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return arc::set_cuda_error(e, "matvec_hostio h2d");
    st = arc::matvec_launch(pl, w, nullptr, x_dev, nullptr, 0.f, nullptr, nullptr, y_dev, s);
    if (st != ARC_OK) return st;
    e = cudaMemcpyAsync(y_host, y_dev, sizeof(float) * rows, cudaMemcpyDeviceToHost, s);
    if (e != cudaSuccess) return arc::set_cuda_error(e, "matvec_hostio d2h");
    e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return arc::set_cuda_error(e, "matvec_hostio sync");
    return ARC_OK;
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
    arc::MatvecPlan pl;
    int st = arc::matvec_plan(ARC_GGML_Q4_K, true, rows, k, &pl);
    if (st != ARC_OK) return st;
    return arc::matvec_launch(pl, w_gate, w_up, x, gamma, eps, nullptr, nullptr, s,
                              static_cast<cudaStream_t>(stream));
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

}  // extern "C"
