// Batched prefill kernels around the tcgen05 GEMMs (B200, sm_100a): the
// per-token elementwise steps of the reference's prefill chain
// (src/arcllm_v1_runtime.cpp:340-369) applied to T prompt rows at once.
//
//   rmsnorm_rows_bf16   y = x * rsqrt(mean(x^2) + eps) * gamma per row, sum of
//                       squares in double (src/p8c_segmented_access_correctness.cpp:958-969,
//                       the same expression the matvecs fuse), rounded to bf16
//                       as the GEMMs' activation operand;
//   rope_kv_rows        + bias, RoPE on q and k and the fp16 KV store for
//                       positions pos0 .. pos0+T-1 (the decode kernel's
//                       arithmetic, so a prompt row lands in the cache as the
//                       token-by-token path would store the same inputs);
//   attention_prefill   causal GQA attention, query row t over positions
//                       0 .. pos0+t of the cache (shaders/p7_attention_prefill_online.comp,
//                       CPU form p8c...:1136-1158), one CTA per (row, KV head)
//                       with the group's q heads in registers and an online
//                       softmax; the result is written as bf16 for the O GEMM;
//   silu_mul_rows_bf16  s = silu(g) * u (p8c...:1064-1073), bf16 for the down GEMM.
#include <algorithm>
#include <cfloat>

#include "arcllm_cuda_internal.h"
#include "common.cuh"
#include "decode_ops.h"
#include "prefill_ops.h"

namespace arc {
namespace {

__device__ __forceinline__ uint16_t f2bf(float f) {
    uint16_t r;
    asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(r) : "f"(f));
    return r;
}

// One CTA (256 threads) per row.
__global__ void __launch_bounds__(256) rmsnorm_rows_bf16_kernel(const float* __restrict__ x,
                                                                const float* __restrict__ gamma, float eps, uint32_t h,
                                                                uint16_t* __restrict__ out) {
    __shared__ double red[8];
    const float* xr = x + (uint64_t)blockIdx.x * h;
    double ss = 0.0;
    for (uint32_t i = threadIdx.x; i < h; i += 256u) {
        const double v = (double)xr[i];
        ss += v * v;
    }
    ss = warp_sum_d(ss);
    if ((threadIdx.x & 31u) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    double tot = 0.0;
#pragma unroll
    for (int w = 0; w < 8; ++w) tot += red[w];
    const float inv = 1.0f / sqrtf((float)(tot / (double)h) + eps);
    uint16_t* o = out + (uint64_t)blockIdx.x * h;
    for (uint32_t i = threadIdx.x; i < h; i += 256u) o[i] = f2bf((xr[i] * inv) * gamma[i]);
}

// One thread per rotation pair of one row: q pairs, then k pairs (with v).
__global__ void rope_kv_rows_kernel(float* __restrict__ q, float* __restrict__ k, const float* __restrict__ v,
                                    const float* __restrict__ bq, const float* __restrict__ bk,
                                    const float* __restrict__ bv, const float2* __restrict__ table, uint32_t pos0,
                                    uint16_t* __restrict__ kc, uint16_t* __restrict__ vc, RopeKvShape s) {
    const uint32_t t = blockIdx.y, pos = pos0 + t;
    const uint32_t half = s.head_dim / 2u;
    const uint32_t nq = s.q_heads * half, nk = s.kv_heads * half;
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t hdim = s.q_heads * s.head_dim, kv_dim = s.kv_heads * s.head_dim;
    const float2* tr = table + (uint64_t)pos * half;
    const uint64_t cbase = ((uint64_t)s.layer * s.max_ctx + pos) * kv_dim;
    if (i < nq) {
        const uint32_t hh = i / half, pp = i - hh * half;
        const uint32_t o = hh * s.head_dim + 2u * pp;
        const float2 cs = tr[pp];
        float* x = q + (uint64_t)t * hdim + o;
        const float a = x[0] + (bq ? bq[o] : 0.f), b = x[1] + (bq ? bq[o + 1] : 0.f);
        x[0] = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
        x[1] = __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x));
    } else if (i < nq + nk) {
        const uint32_t j = i - nq, hh = j / half, pp = j - hh * half;
        const uint32_t o = hh * s.head_dim + 2u * pp;
        const float2 cs = tr[pp];
        float* kx = k + (uint64_t)t * kv_dim + o;
        const float* vx = v + (uint64_t)t * kv_dim + o;
        const float a = kx[0] + (bk ? bk[o] : 0.f), b = kx[1] + (bk ? bk[o + 1] : 0.f);
        const float r0 = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
        const float r1 = __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x));
        kx[0] = r0;
        kx[1] = r1;
        kc[cbase + o] = __half_as_ushort(__float2half_rn(r0));
        kc[cbase + o + 1] = __half_as_ushort(__float2half_rn(r1));
        vc[cbase + o] = __half_as_ushort(__float2half_rn(vx[0] + (bv ? bv[o] : 0.f)));
        vc[cbase + o + 1] = __half_as_ushort(__float2half_rn(vx[1] + (bv ? bv[o + 1] : 0.f)));
    }
}

// Causal attention for query row t (blockIdx.x) and KV head blockIdx.y over
// positions 0 .. pos0+t.  Warps stride over positions; lane L owns head dims
// 4L..4L+3 of all GQ q heads of the group; the 8 warps' online-softmax states
// are combined in shared memory at the end (in warp order).
template <int GQ>
__global__ void __launch_bounds__(256) attention_prefill_kernel(const float* __restrict__ q,
                                                                const uint16_t* __restrict__ kc,
                                                                const uint16_t* __restrict__ vc, uint32_t pos0,
                                                                AttnShape s, uint16_t* __restrict__ out) {
    constexpr int D = 128, NW = 8;
    __shared__ float sm_m[NW][GQ], sm_l[NW][GQ];
    __shared__ float sm_acc[NW][GQ][D];
    const uint32_t t = blockIdx.x, kvh = blockIdx.y;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t n = pos0 + t + 1u;
    const uint32_t hdim = s.q_heads * D, kv_dim = s.kv_heads * D;
    float qv[GQ][4];
#pragma unroll
    for (int g = 0; g < GQ; ++g) {
        const float4 a = *reinterpret_cast<const float4*>(q + (uint64_t)t * hdim + (kvh * GQ + g) * D + lane * 4u);
        qv[g][0] = a.x * s.scale, qv[g][1] = a.y * s.scale, qv[g][2] = a.z * s.scale, qv[g][3] = a.w * s.scale;
    }
    float m[GQ], l[GQ], acc[GQ][4];
#pragma unroll
    for (int g = 0; g < GQ; ++g) {
        m[g] = -FLT_MAX, l[g] = 0.f;
        acc[g][0] = acc[g][1] = acc[g][2] = acc[g][3] = 0.f;
    }
    const uint64_t lbase = (uint64_t)s.layer * s.max_ctx * kv_dim + kvh * D + lane * 4u;
    for (uint32_t p = warp; p < n; p += NW) {
        const uint2 kraw = *reinterpret_cast<const uint2*>(kc + lbase + (uint64_t)p * kv_dim);
        const uint2 vraw = *reinterpret_cast<const uint2*>(vc + lbase + (uint64_t)p * kv_dim);
        const float2 k01 = __half22float2(*reinterpret_cast<const __half2*>(&kraw.x));
        const float2 k23 = __half22float2(*reinterpret_cast<const __half2*>(&kraw.y));
        const float2 v01 = __half22float2(*reinterpret_cast<const __half2*>(&vraw.x));
        const float2 v23 = __half22float2(*reinterpret_cast<const __half2*>(&vraw.y));
        float sc[GQ];
#pragma unroll
        for (int g = 0; g < GQ; ++g)
            sc[g] = fmaf(qv[g][0], k01.x, fmaf(qv[g][1], k01.y, fmaf(qv[g][2], k23.x, qv[g][3] * k23.y)));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
            for (int g = 0; g < GQ; ++g) sc[g] += __shfl_xor_sync(0xffffffffu, sc[g], o);
        }
#pragma unroll
        for (int g = 0; g < GQ; ++g) {
            const float mn = fmaxf(m[g], sc[g]);
            const float a = __expf(m[g] - mn), pr = __expf(sc[g] - mn);
            l[g] = fmaf(l[g], a, pr);
            acc[g][0] = fmaf(acc[g][0], a, pr * v01.x);
            acc[g][1] = fmaf(acc[g][1], a, pr * v01.y);
            acc[g][2] = fmaf(acc[g][2], a, pr * v23.x);
            acc[g][3] = fmaf(acc[g][3], a, pr * v23.y);
            m[g] = mn;
        }
    }
#pragma unroll
    for (int g = 0; g < GQ; ++g) {
        if (lane == 0) sm_m[warp][g] = m[g], sm_l[warp][g] = l[g];
        *reinterpret_cast<float4*>(&sm_acc[warp][g][lane * 4u]) = make_float4(acc[g][0], acc[g][1], acc[g][2], acc[g][3]);
    }
    __syncthreads();
    for (uint32_t idx = threadIdx.x; idx < GQ * D; idx += 256u) {
        const uint32_t g = idx / D, d = idx - g * D;
        float M = -FLT_MAX;
#pragma unroll
        for (int w = 0; w < NW; ++w) M = fmaxf(M, sm_m[w][g]);
        float L = 0.f, Acc = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            const float f = __expf(sm_m[w][g] - M);
            L = fmaf(sm_l[w][g], f, L);
            Acc = fmaf(sm_acc[w][g][d], f, Acc);
        }
        out[(uint64_t)t * hdim + (kvh * GQ + g) * D + d] = f2bf(Acc / L);
    }
}

__global__ void silu_mul_rows_bf16_kernel(const float* __restrict__ g, const float* __restrict__ u, uint64_t n,
                                          uint16_t* __restrict__ out) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        const float a = g[i];
        out[i] = f2bf((a / (1.0f + expf(-a))) * u[i]);
    }
}

// After a batched prefill of positions 0 .. n_prompt-2: the decode graph
// continues with the last prompt token at its position.
__global__ void prefill_done_kernel(GreedyState* st, const uint32_t* __restrict__ prompt, uint32_t n_prompt) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    st->pos = n_prompt - 1u;
    st->token = prompt[n_prompt - 1u];
    st->argmax_key = 0ull;
}

}  // namespace

int launch_prefill_done(GreedyState* st, const uint32_t* prompt, uint32_t n_prompt, cudaStream_t stream) {
    if (n_prompt == 0) return set_error(ARC_E_INVALID_ARGUMENT, "prefill: empty prompt");
    return launch_checked(launch_kernel(prefill_done_kernel, dim3(1), dim3(32), 0, stream, st, prompt, n_prompt),
                          "prefill done launch");
}

int launch_rmsnorm_rows_bf16(const float* x, const float* gamma, float eps, uint32_t rows, uint32_t h, uint16_t* out,
                             cudaStream_t stream) {
    if (rows == 0) return ARC_OK;
    return launch_checked(
        launch_kernel(rmsnorm_rows_bf16_kernel, dim3(rows), dim3(256), 0, stream, x, gamma, eps, h, out),
        "rmsnorm rows launch");
}

int launch_rope_kv_rows(float* q, float* k, const float* v, const float* bq, const float* bk, const float* bv,
                        const float2* table, uint32_t pos0, uint32_t rows, uint16_t* kc, uint16_t* vc,
                        const RopeKvShape& s, cudaStream_t stream) {
    if (rows == 0) return ARC_OK;
    if (pos0 + rows > s.max_ctx) return set_error(ARC_E_INVALID_ARGUMENT, "rope rows: positions past the context");
    const uint32_t pairs = (s.q_heads + s.kv_heads) * (s.head_dim / 2u);
    return launch_checked(launch_kernel(rope_kv_rows_kernel, dim3((pairs + 127) / 128, rows), dim3(128), 0, stream, q,
                                        k, v, bq, bk, bv, table, pos0, kc, vc, s),
                          "rope rows launch");
}

int launch_attention_prefill(const float* q, const uint16_t* kc, const uint16_t* vc, uint32_t pos0, uint32_t rows,
                             const AttnShape& s, uint16_t* out, cudaStream_t stream) {
    if (rows == 0) return ARC_OK;
    if (s.head_dim != 128u) return set_error(ARC_E_UNSUPPORTED_SHAPE, "attention: head_dim must be 128");
    if (pos0 + rows > s.max_ctx) return set_error(ARC_E_INVALID_ARGUMENT, "attention: positions past the context");
    const uint32_t gq = s.q_heads / s.kv_heads;
    if (gq * s.kv_heads != s.q_heads) return set_error(ARC_E_UNSUPPORTED_SHAPE, "attention: q_heads % kv_heads");
    const dim3 grid(rows, s.kv_heads);
    cudaError_t e;
    switch (gq) {
        case 1: e = launch_kernel(attention_prefill_kernel<1>, grid, dim3(256), 0, stream, q, kc, vc, pos0, s, out); break;
        case 2: e = launch_kernel(attention_prefill_kernel<2>, grid, dim3(256), 0, stream, q, kc, vc, pos0, s, out); break;
        case 4: e = launch_kernel(attention_prefill_kernel<4>, grid, dim3(256), 0, stream, q, kc, vc, pos0, s, out); break;
        case 7: e = launch_kernel(attention_prefill_kernel<7>, grid, dim3(256), 0, stream, q, kc, vc, pos0, s, out); break;
        case 8: e = launch_kernel(attention_prefill_kernel<8>, grid, dim3(256), 0, stream, q, kc, vc, pos0, s, out); break;
        default: return set_error(ARC_E_UNSUPPORTED_SHAPE, "attention: q heads per kv head must be 1, 2, 4, 7 or 8");
    }
    return launch_checked(e, "attention prefill launch");
}

int launch_silu_mul_rows_bf16(const float* g, const float* u, uint64_t n, uint16_t* out, cudaStream_t stream) {
    if (n == 0) return ARC_OK;
    const uint32_t blocks = (uint32_t)std::min<uint64_t>((n + 255) / 256, 148u * 16u);
    return launch_checked(launch_kernel(silu_mul_rows_bf16_kernel, dim3(blocks), dim3(256), 0, stream, g, u, n, out),
                          "silu mul launch");
}

}  // namespace arc
