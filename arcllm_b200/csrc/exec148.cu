// EXEC148: the re-laid-out Q4_K image of the FFN-down weights (primitive B of
// the reference's Q4 down capability).  One 148-byte block per Q4_K
// super-block: d and dmin (4 bytes, copied), the eight 6-bit (scale, min)
// pairs unpacked to one byte each (16 bytes), then the 256 codes as 128
// nibble pairs in element order (byte p = q[2p] | q[2p+1] << 4), so the codes
// of sub-block j are the 16 contiguous bytes 20 + 16j .. 35 + 16j.
//
//   materialize  src/q4_down_exec148_materializer.h:14 (materialize_block),
//                shaders/b1_2_exec148_gpu_materialize.comp:44-75 (P1, on the GPU)
//   validate     src/q4_down_exec148_materializer.h:16-18 (canonical tuples:
//                d, dmin, 8 x (sc, mn), 256 codes -- identical for source and image)
//   matvec       shaders/q4_down_exec148_serial.comp:6 (y = W x with the same
//                w = d*sc*q - dmin*mn per element)
#include <algorithm>
#include <atomic>

#include "arcllm_cuda_internal.h"
#include "common.cuh"

namespace arc {
namespace {

// (scale, min) of sub-block j from the 12 packed bytes s[0..11] (block bytes 4..15):
// src/p8c_segmented_access_correctness.cpp:531-540
__device__ __forceinline__ void q4k_scale_min(const uint8_t* s, uint32_t j, uint32_t& sc, uint32_t& mn) {
    if (j < 4) {
        sc = s[j] & 63u;
        mn = s[j + 4] & 63u;
    } else {
        sc = (s[j + 4] & 15u) | ((s[j - 4] >> 6) << 4);
        mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

// element k (0..255) of a Q4_K super-block's codes
__device__ __forceinline__ uint32_t q4k_code(const uint8_t* blk, uint32_t k) {
    const uint32_t x = k & 63u;
    const uint32_t b = blk[16u + (k >> 6) * 32u + (x & 31u)];
    return x < 32u ? (b & 15u) : (b >> 4);
}

__global__ void exec148_materialize_kernel(const uint8_t* __restrict__ src, uint64_t n_blocks,
                                           uint8_t* __restrict__ dst) {
    pdl_trigger();
    pdl_wait();
    const uint64_t b = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= n_blocks) return;
    uint8_t s[144];
#pragma unroll
    for (int i = 0; i < 9; ++i) *reinterpret_cast<uint4*>(s + 16 * i) = ld_nc_v4(src + b * 144u + 16u * i);
    uint32_t out[37];
    out[0] = (uint32_t)s[0] | ((uint32_t)s[1] << 8) | ((uint32_t)s[2] << 16) | ((uint32_t)s[3] << 24);
#pragma unroll
    for (uint32_t w = 0; w < 4; ++w) {
        uint32_t sc0, mn0, sc1, mn1;
        q4k_scale_min(s + 4, 2u * w, sc0, mn0);
        q4k_scale_min(s + 4, 2u * w + 1u, sc1, mn1);
        out[1 + w] = sc0 | (mn0 << 8) | (sc1 << 16) | (mn1 << 24);
    }
#pragma unroll
    for (uint32_t w = 0; w < 32; ++w) {
        uint32_t v = 0;
#pragma unroll
        for (uint32_t i = 0; i < 4; ++i) {
            const uint32_t p = 4u * w + i;
            v |= (q4k_code(s, 2u * p) | (q4k_code(s, 2u * p + 1u) << 4)) << (8u * i);
        }
        out[5 + w] = v;
    }
    uint32_t* d = reinterpret_cast<uint32_t*>(dst + b * 148u);  // 148 = 4 x 37: 4-byte aligned
#pragma unroll
    for (int i = 0; i < 37; ++i) d[i] = out[i];
}

// Count blocks whose canonical tuple (d, dmin, 8 x (sc, mn), 256 codes) differs
// between the Q4_K source and the EXEC148 image.
__global__ void exec148_validate_kernel(const uint8_t* __restrict__ src, const uint8_t* __restrict__ img,
                                        uint64_t n_blocks, unsigned long long* mismatches) {
    pdl_trigger();
    pdl_wait();
    const uint64_t b = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= n_blocks) return;
    const uint8_t* s = src + b * 144u;
    const uint8_t* e = img + b * 148u;
    bool same = s[0] == e[0] && s[1] == e[1] && s[2] == e[2] && s[3] == e[3];
    for (uint32_t j = 0; j < 8; ++j) {
        uint32_t sc, mn;
        q4k_scale_min(s + 4, j, sc, mn);
        same = same && sc == e[4 + 2 * j] && mn == e[5 + 2 * j];
    }
    for (uint32_t k = 0; k < 256; ++k) {
        const uint32_t p = e[20u + (k >> 1)];
        same = same && q4k_code(s, k) == ((k & 1u) ? (p >> 4) : (p & 15u));
    }
    if (!same) atomicAdd(mismatches, 1ull);
}

// y[r] = (residual[r] +) sum_k w[r,k] x[k] over EXEC148 rows.  Persistent
// CTAs stage x and the per-sub-block sums of x in shared memory once; each
// warp then takes rows in turn, lane L sub-blocks L, L+32, ... of the row,
// loading kExecUnroll sub-blocks before using any (bytes in flight).
// A code q enters as the float 1 + q/16 (its nibble placed in the mantissa):
// sum(q x) = 16 (sum((1 + q/16) x) - sum(x)), and per sub-block
// sum(w x) = d sc sum(q x) - dmin mn sum(x).
constexpr uint32_t kExecWarps = 16;
constexpr uint32_t kExecUnroll = 4;

__global__ void __launch_bounds__(kExecWarps * 32, 2) exec148_matvec_kernel(const uint8_t* __restrict__ w,
                                                                            uint32_t rows, uint32_t k,
                                                                            const float* __restrict__ x,
                                                                            const float* __restrict__ residual,
                                                                            float* __restrict__ y) {
    extern __shared__ __align__(16) float xs[];  // [k] x, then [k/32] sub-block sums
    float* sxs = xs + k;
    pdl_trigger();
    pdl_wait();
    const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
    const uint32_t nsub = k / 32u;
    for (uint32_t i = tid; i < k / 4u; i += blockDim.x)
        reinterpret_cast<float4*>(xs)[i] = reinterpret_cast<const float4*>(x)[i];
    __syncthreads();
    for (uint32_t j = tid; j < nsub; j += blockDim.x) {
        float t = 0.f;
        for (uint32_t e = 0; e < 32; ++e) t += xs[32u * j + e];
        sxs[j] = t;
    }
    __syncthreads();
    const uint64_t rb = (uint64_t)(k / 256u) * 148u;
    for (uint32_t row = blockIdx.x * kExecWarps + warp; row < rows; row += gridDim.x * kExecWarps) {
        const uint8_t* rp = w + row * rb;
        float acc = 0.f;
        for (uint32_t j0 = lane; j0 < nsub; j0 += 32u * kExecUnroll) {
            uint32_t c[kExecUnroll][4], hd[kExecUnroll], scmn[kExecUnroll];
#pragma unroll
            for (uint32_t u = 0; u < kExecUnroll; ++u) {
                const uint32_t j = j0 + 32u * u;
                if (j < nsub) {
                    const uint8_t* blk = rp + (j >> 3) * 148u;
                    const uint32_t jj = j & 7u;
                    // blocks are 148 bytes apart, so the codes are only 4-byte aligned
                    const uint32_t* cp = reinterpret_cast<const uint32_t*>(blk + 20u + 16u * jj);
#pragma unroll
                    for (int i = 0; i < 4; ++i) c[u][i] = __ldg(cp + i);
                    hd[u] = __ldg(reinterpret_cast<const uint32_t*>(blk));
                    scmn[u] = __ldg(reinterpret_cast<const unsigned short*>(blk + 4u + 2u * jj));
                } else {
                    c[u][0] = c[u][1] = c[u][2] = c[u][3] = 0u;
                    hd[u] = scmn[u] = 0u;
                }
            }
#pragma unroll
            for (uint32_t u = 0; u < kExecUnroll; ++u) {
                const uint32_t j = j0 + 32u * u;
                if (j >= nsub) break;
                const float4* xv = reinterpret_cast<const float4*>(xs + 32u * j);
                float t = 0.f;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float4 xa = xv[2 * i], xb = xv[2 * i + 1];
                    const float xe[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const int bit = 4 * e;  // nibble e of the word -> mantissa bits 19..22
                        const uint32_t m = bit <= 19 ? (c[u][i] << (19 - bit)) : (c[u][i] >> (bit - 19));
                        t = fmaf(__uint_as_float((m & 0x00780000u) | 0x3F800000u), xe[e], t);
                    }
                }
                const float d = __half2float(__ushort_as_half((unsigned short)(hd[u] & 0xFFFFu)));
                const float dmin = __half2float(__ushort_as_half((unsigned short)(hd[u] >> 16)));
                const float sx = sxs[j];
                const float qx = 16.0f * (t - sx);
                acc = fmaf(d * (float)(scmn[u] & 0xFFu), qx, fmaf(-(dmin * (float)(scmn[u] >> 8)), sx, acc));
            }
        }
        acc = warp_sum(acc);
        if (lane == 0) y[row] = residual ? residual[row] + acc : acc;
    }
}

}  // namespace

int exec148_materialize(const void* src, uint64_t n_blocks, void* dst, cudaStream_t stream) {
    if (!src || !dst) return set_error(ARC_E_INVALID_ARGUMENT, "exec148_materialize: null pointer");
    if ((reinterpret_cast<uintptr_t>(src) & 15u) || (reinterpret_cast<uintptr_t>(dst) & 3u))
        return set_error(ARC_E_ALIGNMENT, "exec148_materialize: source 16-byte, image 4-byte alignment");
    if (n_blocks == 0) return ARC_OK;
    const cudaError_t e = launch_kernel(exec148_materialize_kernel, dim3((unsigned)((n_blocks + 127) / 128)),
                                        dim3(128), 0, stream, static_cast<const uint8_t*>(src), n_blocks,
                                        static_cast<uint8_t*>(dst));
    return e == cudaSuccess ? ARC_OK : set_cuda_error(e, "exec148_materialize launch");
}

int exec148_validate(const void* src, const void* img, uint64_t n_blocks, uint64_t* mismatches_host,
                     cudaStream_t stream) {
    if (!src || !img || !mismatches_host) return set_error(ARC_E_INVALID_ARGUMENT, "exec148_validate: null pointer");
    if (reinterpret_cast<uintptr_t>(img) & 3u) return set_error(ARC_E_ALIGNMENT, "exec148_validate: image alignment");
    unsigned long long* dcount = nullptr;
    cudaError_t e = cudaMallocAsync(&dcount, sizeof(unsigned long long), stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(dcount, 0, sizeof(unsigned long long), stream);
    if (e == cudaSuccess && n_blocks)
        e = launch_kernel(exec148_validate_kernel, dim3((unsigned)((n_blocks + 127) / 128)), dim3(128), 0, stream,
                          static_cast<const uint8_t*>(src), static_cast<const uint8_t*>(img), n_blocks, dcount);
    unsigned long long h = 0;
    if (e == cudaSuccess) e = cudaMemcpyAsync(&h, dcount, sizeof h, cudaMemcpyDeviceToHost, stream);
    if (dcount) cudaFreeAsync(dcount, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return set_cuda_error(e, "exec148_validate");
    *mismatches_host = h;
    return ARC_OK;
}

int exec148_matvec(const void* w, uint32_t rows, uint32_t k, const float* x, const float* residual, float* y,
                   cudaStream_t stream) {
    if (!w || !x || !y) return set_error(ARC_E_INVALID_ARGUMENT, "matvec: null pointer");
    if (rows == 0 || k == 0 || k % 256u) return set_error(ARC_E_UNSUPPORTED_SHAPE, "matvec: K must be a multiple of 256");
    if ((reinterpret_cast<uintptr_t>(w) & 3u) || (reinterpret_cast<uintptr_t>(x) & 15u))
        return set_error(ARC_E_ALIGNMENT, "matvec EXEC148: image 4-byte, x 16-byte aligned");
    const size_t smem = (size_t)k * 4u + (size_t)(k / 32u) * 4u;
    if (smem > 227u * 1024u) return set_error(ARC_E_UNSUPPORTED_SHAPE, "matvec EXEC148: K too large");
    static std::atomic<bool> attr_done[64] = {};  // concurrent first calls set the same (idempotent) attribute
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    const int slot = device_slot();
    if (slot < 0) return set_error(ARC_E_CUDA, "matvec EXEC148: no current device below index 64");
    if (!attr_done[slot].load(std::memory_order_acquire)) {
        const cudaError_t a = cudaFuncSetAttribute(exec148_matvec_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   227 * 1024);
        if (a != cudaSuccess) return set_cuda_error(a, "matvec EXEC148 attribute");
        attr_done[slot].store(true, std::memory_order_release);
    }
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const uint32_t per_sm = smem <= 113u * 1024u ? 2u : 1u;
    const uint32_t grid = std::min<uint32_t>((rows + kExecWarps - 1) / kExecWarps, (uint32_t)sms * per_sm);
    const cudaError_t e = launch_kernel(exec148_matvec_kernel, dim3(grid), dim3(kExecWarps * 32), smem, stream,
                                        static_cast<const uint8_t*>(w), rows, k, x, residual, y);
    return e == cudaSuccess ? ARC_OK : set_cuda_error(e, "matvec EXEC148 launch");
}

}  // namespace arc
