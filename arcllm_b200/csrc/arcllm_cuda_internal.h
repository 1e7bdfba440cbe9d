// Internal declarations shared by the CUDA translation units of
// libarcllm_cuda.so.  Nothing here crosses the C ABI (include/arcllm_cuda.h).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/arcllm_cuda.h"

namespace arc {

// Record a status + message for arcllm_cuda_last_error_message(); returns status.
int set_error(int status, const char* msg);
int set_cuda_error(cudaError_t e, const char* where);

// Device address of this library's device error word on the current device
// (nullptr if it cannot be resolved).
unsigned int* dev_error_word();

struct MatvecPlan {
    int fmt = 0;
    bool dual = false;
    uint32_t rows = 0, k = 0, nb = 0, rb = 0;
    uint32_t G = 0, gmax = 0, n_groups = 0, stages = 0, stage_smem = 0, x_floats = 0;
    uint32_t smem = 0, grid = 0;
};

int matvec_plan(int fmt, bool dual, uint32_t rows, uint32_t k, MatvecPlan* out);
int matvec_launch(const MatvecPlan& pl, const void* w0, const void* w1, const float* x, const float* gamma,
                  float eps, const float* bias, const float* residual, float* y, cudaStream_t stream);

}  // namespace arc
