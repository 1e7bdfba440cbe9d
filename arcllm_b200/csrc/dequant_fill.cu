// Bit-exact super-block dequantisation and the synthetic fixture generators.
//
// dequant: one CTA of 256 threads per super-block, element k on thread k,
// computed with separately rounded fp32 operations in the reference's order
// (src/p8c_segmented_access_correctness.cpp:1166-1181 for Q4_K,
// :905-956 for Q6_K) -- no FMA contraction, so the values are identical to
// the reference's CPU dequantisation bit for bit.
//
// fill: element n of the splitmix64 sequence of `seed` is
// mix(seed + (n+1)*0x9E3779B97F4A7C15) (the sequential generator of
// src/sa1_component_benchmark.cpp:71-76 evaluated at call n+1), so any block
// of a tensor can be generated independently.  Field layout per block:
//   Q4_K block i uses words 20i..20i+19: w0 -> d = fp16(1e-3 + 3e-3*u24),
//     w1 -> dmin = fp16(2e-3*u24), w2/w3 -> sixteen 6-bit values (8 scales,
//     8 mins) packed into the 12-byte K-quant scale layout, w4..w19 -> the
//     128 nibble bytes;
//   Q6_K block i uses words 27i..27i+26: w0..w23 -> ql/qh bytes,
//     w24/w25 -> sixteen 6-bit values v, scale = v - 32, w26 -> d.
// The same arithmetic is restated on the CPU in the test oracle.
#include "arcllm_cuda_internal.h"
#include "common.cuh"

namespace arc {
namespace {

__device__ __forceinline__ uint16_t ld_u16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

__global__ void dequant_q4k_kernel(const uint8_t* __restrict__ w, uint64_t n_blocks, float* __restrict__ y) {
    const uint64_t ib = blockIdx.x;
    if (ib >= n_blocks) return;
    const uint8_t* b = w + ib * 144u;
    const uint32_t k = threadIdx.x;
    const float d = half_bits_to_float(ld_u16(b));
    const float dmin = half_bits_to_float(ld_u16(b + 2));
    const uint8_t* q = b + 4;
    const uint32_t j = k >> 5;
    uint32_t sc, mn;
    if (j < 4) {
        sc = q[j] & 63u;
        mn = q[j + 4] & 63u;
    } else {
        sc = (q[j + 4] & 0xFu) | ((q[j - 4] >> 6) << 4);
        mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
    const uint32_t g = k >> 6, l = k & 63u;
    const uint8_t qb = b[16u + g * 32u + (l & 31u)];
    const uint32_t qv = l < 32u ? (qb & 15u) : (qb >> 4);
    const float a = __fmul_rn(__fmul_rn(d, (float)sc), (float)qv);
    y[ib * 256u + k] = __fsub_rn(a, __fmul_rn(dmin, (float)mn));
}

__global__ void dequant_q6k_kernel(const uint8_t* __restrict__ w, uint64_t n_blocks, float* __restrict__ y) {
    const uint64_t ib = blockIdx.x;
    if (ib >= n_blocks) return;
    const uint8_t* b = w + ib * 210u;
    const uint32_t k = threadIdx.x;
    const uint32_t half = k >> 7, kk = k & 127u, l = kk & 31u, quarter = kk >> 5;
    const uint8_t* ql = b + half * 64u;
    const uint8_t* qh = b + 128u + half * 32u;
    const uint8_t* scp = b + 192u + half * 8u;
    const uint32_t is = l >> 4;
    uint32_t low, high, si;
    if (quarter == 0u) {
        low = ql[l] & 15u; high = qh[l] & 3u; si = is;
    } else if (quarter == 1u) {
        low = ql[l + 32u] & 15u; high = (qh[l] >> 2) & 3u; si = is + 2u;
    } else if (quarter == 2u) {
        low = ql[l] >> 4; high = (qh[l] >> 4) & 3u; si = is + 4u;
    } else {
        low = ql[l + 32u] >> 4; high = (qh[l] >> 6) & 3u; si = is + 6u;
    }
    const int scv = (int)(int8_t)scp[si];
    const int qv = (int)(low | (high << 4)) - 32;
    const float d = half_bits_to_float(ld_u16(b + 208));
    y[ib * 256u + k] = __fmul_rn(__fmul_rn(d, (float)scv), (float)qv);
}

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ uint64_t sm_at(uint64_t seed, uint64_t n) {
    return mix64(seed + (n + 1u) * 0x9E3779B97F4A7C15ull);
}

__device__ __forceinline__ float unit24(uint64_t w) {
    return __fmul_rn(__uint2float_rn((uint32_t)(w >> 40)), 5.9604644775390625e-08f);
}

__device__ __forceinline__ uint32_t f2h_bits(float f) { return (uint32_t)__half_as_ushort(__float2half_rn(f)); }

__global__ void fill_q4k_kernel(uint8_t* __restrict__ dst, uint64_t block_begin, uint64_t n_blocks, uint64_t seed) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_blocks) return;
    const uint64_t base = (block_begin + i) * 20u;
    uint32_t* o = reinterpret_cast<uint32_t*>(dst + i * 144u);
    const uint64_t w0 = sm_at(seed, base), w1 = sm_at(seed, base + 1);
    const float d = __fadd_rn(1e-3f, __fmul_rn(3e-3f, unit24(w0)));
    const float dmin = __fmul_rn(2e-3f, unit24(w1));
    o[0] = f2h_bits(d) | (f2h_bits(dmin) << 16);
    const uint64_t w2 = sm_at(seed, base + 2), w3 = sm_at(seed, base + 3);
    uint32_t v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = (uint32_t)(j < 10 ? (w2 >> (6 * j)) & 63u : (w3 >> (6 * (j - 10))) & 63u);
    uint8_t q[12];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        q[j] = (uint8_t)((v[j] & 63u) | ((v[j + 4] >> 4) << 6));
        q[j + 4] = (uint8_t)((v[8 + j] & 63u) | ((v[8 + j + 4] >> 4) << 6));
    }
#pragma unroll
    for (int j = 4; j < 8; ++j) q[j + 4] = (uint8_t)((v[j] & 15u) | ((v[8 + j] & 15u) << 4));
#pragma unroll
    for (int t = 0; t < 3; ++t)
        o[1 + t] = (uint32_t)q[4 * t] | ((uint32_t)q[4 * t + 1] << 8) | ((uint32_t)q[4 * t + 2] << 16) |
                   ((uint32_t)q[4 * t + 3] << 24);
#pragma unroll
    for (int t = 0; t < 16; ++t) {
        const uint64_t wq = sm_at(seed, base + 4 + t);
        o[4 + 2 * t] = (uint32_t)wq;
        o[5 + 2 * t] = (uint32_t)(wq >> 32);
    }
}

__global__ void fill_q6k_kernel(uint8_t* __restrict__ dst, uint64_t block_begin, uint64_t n_blocks, uint64_t seed) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_blocks) return;
    const uint64_t base = (block_begin + i) * 27u;
    uint16_t* o = reinterpret_cast<uint16_t*>(dst + i * 210u);  // 2-byte aligned for every block
#pragma unroll 4
    for (int t = 0; t < 24; ++t) {
        const uint64_t wq = sm_at(seed, base + t);
#pragma unroll
        for (int h = 0; h < 4; ++h) o[4 * t + h] = (uint16_t)(wq >> (16 * h));
    }
    const uint64_t w24 = sm_at(seed, base + 24), w25 = sm_at(seed, base + 25);
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
        const uint32_t a = (uint32_t)(j < 10 ? (w24 >> (6 * j)) & 63u : (w25 >> (6 * (j - 10))) & 63u);
        const uint32_t b = (uint32_t)(j + 1 < 10 ? (w24 >> (6 * (j + 1))) & 63u : (w25 >> (6 * (j + 1 - 10))) & 63u);
        const uint32_t sa = (uint32_t)(uint8_t)(int8_t)((int)a - 32), sb = (uint32_t)(uint8_t)(int8_t)((int)b - 32);
        o[96 + j / 2] = (uint16_t)(sa | (sb << 8));
    }
    const float d = __fadd_rn(1e-3f, __fmul_rn(3e-3f, unit24(sm_at(seed, base + 26))));
    o[104] = (uint16_t)f2h_bits(d);
}

__device__ __forceinline__ float ih_normal(uint64_t w, float mu, float sigma) {
    const int32_t s = (int32_t)((w & 0xffffu) + ((w >> 16) & 0xffffu) + ((w >> 32) & 0xffffu) + (w >> 48));
    const float z = __fmul_rn((float)(s - 131070), 1.7320508075688772f * 1.52587890625e-05f);
    return __fadd_rn(mu, __fmul_rn(sigma, z));
}

__global__ void fill_normal_f32_kernel(float* y, uint64_t begin, uint64_t n, uint64_t seed, float mu, float sigma) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = ih_normal(sm_at(seed, begin + i), mu, sigma);
}

__global__ void fill_normal_f16_kernel(uint16_t* y, uint64_t begin, uint64_t n, uint64_t seed, float mu,
                                       float sigma) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = (uint16_t)f2h_bits(ih_normal(sm_at(seed, begin + i), mu, sigma));
}

inline unsigned grid_for(uint64_t n, unsigned threads) { return (unsigned)((n + threads - 1) / threads); }

}  // namespace

int dequant(int fmt, const void* w, uint64_t n_blocks, float* y, cudaStream_t stream) {
    if (!w || !y) return set_error(ARC_E_INVALID_ARGUMENT, "dequant: null pointer");
    if (n_blocks == 0) return ARC_OK;
    if (n_blocks > 0x7fffffffull) return set_error(ARC_E_UNSUPPORTED_SHAPE, "dequant: too many blocks");
    if (fmt == 12)
        dequant_q4k_kernel<<<(unsigned)n_blocks, 256, 0, stream>>>(static_cast<const uint8_t*>(w), n_blocks, y);
    else
        dequant_q6k_kernel<<<(unsigned)n_blocks, 256, 0, stream>>>(static_cast<const uint8_t*>(w), n_blocks, y);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ARC_OK : set_cuda_error(e, "dequant launch");
}

int fill_blocks(int fmt, void* w, uint64_t block_begin, uint64_t n_blocks, uint64_t seed, cudaStream_t stream) {
    if (!w) return set_error(ARC_E_INVALID_ARGUMENT, "fill: null pointer");
    if (n_blocks == 0) return ARC_OK;
    if (fmt == 12) {
        if (reinterpret_cast<uintptr_t>(w) & 3u) return set_error(ARC_E_ALIGNMENT, "fill_q4k: 4-byte alignment");
        fill_q4k_kernel<<<grid_for(n_blocks, 256), 256, 0, stream>>>(static_cast<uint8_t*>(w), block_begin,
                                                                     n_blocks, seed);
    } else {
        if (reinterpret_cast<uintptr_t>(w) & 1u) return set_error(ARC_E_ALIGNMENT, "fill_q6k: 2-byte alignment");
        fill_q6k_kernel<<<grid_for(n_blocks, 256), 256, 0, stream>>>(static_cast<uint8_t*>(w), block_begin,
                                                                     n_blocks, seed);
    }
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ARC_OK : set_cuda_error(e, "fill launch");
}

int fill_normal(bool f16, void* y, uint64_t begin, uint64_t n, uint64_t seed, float mu, float sigma,
                cudaStream_t stream) {
    if (!y) return set_error(ARC_E_INVALID_ARGUMENT, "fill_normal: null pointer");
    if (n == 0) return ARC_OK;
    if (f16)
        fill_normal_f16_kernel<<<grid_for(n, 256), 256, 0, stream>>>(static_cast<uint16_t*>(y), begin, n, seed, mu,
                                                                     sigma);
    else
        fill_normal_f32_kernel<<<grid_for(n, 256), 256, 0, stream>>>(static_cast<float*>(y), begin, n, seed, mu,
                                                                     sigma);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ARC_OK : set_cuda_error(e, "fill_normal launch");
}

}  // namespace arc
