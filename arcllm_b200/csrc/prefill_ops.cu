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
//                       CPU form p8c...:1136-1158) on the tensor cores: per
//                       warp a 16-row tile of (query row, q head) pairs of one
//                       KV head, flash-attention style over 16-position tiles
//                       of the cache; the result is written as bf16 for the O GEMM;
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

// One CTA (256 threads) per row; bf16 output, or fp16 when FP16 (values that
// round to +-inf in fp16 raise the device error word's range bit).
template <bool FP16>
__global__ void __launch_bounds__(256) rmsnorm_rows_bf16_kernel(const float* __restrict__ x,
                                                                const float* __restrict__ gamma, float eps, uint32_t h,
                                                                uint16_t* __restrict__ out,
                                                                uint16_t* __restrict__ out_lo, unsigned int* err) {
    pdl_wait();  // inputs come from the preceding kernels (a no-op for a plain launch)
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
    uint16_t* ol = out_lo ? out_lo + (uint64_t)blockIdx.x * h : nullptr;
    bool range = false;
    for (uint32_t i = threadIdx.x; i < h; i += 256u) {
        const float v = (xr[i] * inv) * gamma[i];
        if (FP16) {
            const __half hv = __float2half_rn(v);
            range |= __hisinf(hv) != 0 && isfinite(v);
            o[i] = __half_as_ushort(hv);
            if (ol) ol[i] = __half_as_ushort(__float2half_rn(v - __half2float(hv)));
        } else {
            o[i] = f2bf(v);
        }
    }
    if (FP16 && range) raise_error(err, ARC_DEV_ERR_RANGE);
}

// One thread per rotation pair of one row: q pairs, then k pairs (with v).
__global__ void rope_kv_rows_kernel(float* __restrict__ q, float* __restrict__ k, const float* __restrict__ v,
                                    const float* __restrict__ bq, const float* __restrict__ bk,
                                    const float* __restrict__ bv, const float2* __restrict__ table, uint32_t pos0,
                                    uint16_t* __restrict__ kc, uint16_t* __restrict__ vc, RopeKvShape s) {
    pdl_wait();  // inputs come from the preceding kernels
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

// D += A * B, m16n8k16, fp16 operands, fp32 accumulators
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_addr(p)));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_addr(p)));
}

__device__ __forceinline__ uint32_t pack_f16(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// 16-byte global -> shared copy that bypasses L1 (cp.async, completion by group)
__device__ __forceinline__ void cp_async_16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Causal attention of query rows r over cache positions 0 .. pos0+r on the
// tensor cores (flash-attention tiling).  A warp owns a 16-row A tile: RQ
// consecutive query rows x the GQ q heads of KV head blockIdx.y (GQ = 7 is
// padded to 8 rows per query row).  It walks the positions in tiles of 16:
// K and V tiles are copied into shared memory with cp.async (two buffers,
// the next tile in flight while this one is used), S = Q K^T comes from
// ldmatrix B fragments and m16n8k16 MMAs, the online softmax runs on the S
// fragments, and O += P V takes P straight from those registers with V
// fragments from ldmatrix.trans.  Q enters as a pair of fp16 halves (q*scale
// = hi + lo), so S is exact to about 2^-22 of |q| |k| (the cache is fp16
// already): scores of the near-one-hot synthetic models stay as sharp as in
// fp32.  P enters the P V product as fp16 (11 bits, the output is bf16).
// |q| * scale must stay inside the fp16 range (< 65504); an element beyond it
// raises the device error word's range bit (its row's output is then not
// meaningful).
template <int GQ>
__global__ void __launch_bounds__(64) attention_prefill_kernel(const float* __restrict__ q,
                                                               const uint16_t* __restrict__ kc,
                                                               const uint16_t* __restrict__ vc, uint32_t pos0,
                                                               uint32_t T, AttnShape s, uint16_t* __restrict__ out,
                                                               unsigned int* err) {
    pdl_wait();  // inputs come from the preceding kernels
    constexpr int D = 128, GP = GQ == 7 ? 8 : GQ, RQ = 16 / GP, NWARP = 2, PT = 16;
    constexpr uint32_t ROWB = D * 2 + 16;  // bytes per cached row in smem (padding: conflict-free ldmatrix)
    __shared__ __align__(128) uint8_t sm[NWARP][2][2][PT * ROWB];  // [warp][buffer][K, V][position row]
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u, g = lane >> 2, t = lane & 3u;
    const uint32_t r0 = (blockIdx.x * NWARP + warp) * RQ;
    if (r0 >= T) return;  // warp-level work only: no CTA barrier below
    const uint32_t kvh = blockIdx.y, hdim = s.q_heads * D, kv_dim = s.kv_heads * D;
    const uint32_t p_hi = pos0 + min(r0 + (uint32_t)RQ, T) - 1u;  // last position this warp's rows see
    // rows g and g + 8 of the A tile
    uint32_t qrow[2], head[2], lim[2];
    bool valid[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint32_t ri = g + 8u * h, qr = r0 + ri / GP;
        head[h] = ri % GP;
        valid[h] = head[h] < (uint32_t)GQ && qr < T;
        qrow[h] = min(qr, T - 1u);
        lim[h] = pos0 + qrow[h];
    }
    // Q fragments, hi and lo fp16 halves of q * scale; register h + 2j of k-step kk holds
    // row g + 8h, dims 16kk + 2t + 8j, +1
    uint32_t qa[8][4], qb[8][4];
    bool range = false;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                float2 v = make_float2(0.f, 0.f);
                if (valid[h])
                    v = *reinterpret_cast<const float2*>(q + (uint64_t)qrow[h] * hdim + (kvh * GQ + head[h]) * D +
                                                         16u * kk + 2u * t + 8u * j);
                v.x *= s.scale, v.y *= s.scale;
                const __half2 hi = __floats2half2_rn(v.x, v.y);
                const float2 hf = __half22float2(hi);
                range |= (isinf(hf.x) && isfinite(v.x)) || (isinf(hf.y) && isfinite(v.y));
                qa[kk][h + 2 * j] = *reinterpret_cast<const uint32_t*>(&hi);
                qb[kk][h + 2 * j] = pack_f16(v.x - hf.x, v.y - hf.y);
            }
    if (range) raise_error(err, ARC_DEV_ERR_RANGE);
    float o[16][4];
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
    const uint64_t lbase = (uint64_t)s.layer * s.max_ctx * kv_dim + kvh * D;
    auto issue = [&](uint32_t tile, int buf) {  // K and V rows of positions tile*16 .. +15 (clamped)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t c = lane + 32u * j, row = c >> 4, ch = c & 15u;
            const uint32_t pos = min(tile * PT + row, p_hi);
            const uint64_t src = lbase + (uint64_t)pos * kv_dim + ch * 8u;
            cp_async_16(&sm[warp][buf][0][row * ROWB + ch * 16u], kc + src);
            cp_async_16(&sm[warp][buf][1][row * ROWB + ch * 16u], vc + src);
        }
        cp_async_commit();
    };
    const uint32_t ntiles = p_hi / PT + 1u;
    issue(0, 0);
    for (uint32_t tile = 0; tile < ntiles; ++tile) {
        const int buf = tile & 1u;
        if (tile + 1u < ntiles) {
            issue(tile + 1u, buf ^ 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncwarp();
        const uint8_t* Ks = sm[warp][buf][0];
        const uint8_t* Vs = sm[warp][buf][1];
        const uint32_t mi = lane >> 3, mr = lane & 7u;  // ldmatrix: matrix and row this lane addresses
        // S in four independent accumulator chains (position block x hi/lo half of q), summed after
        float sc[2][4], sl[2][4];
#pragma unroll
        for (int pb = 0; pb < 2; ++pb) {
            sc[pb][0] = sc[pb][1] = sc[pb][2] = sc[pb][3] = 0.f;
            sl[pb][0] = sl[pb][1] = sl[pb][2] = sl[pb][3] = 0.f;
#pragma unroll
            for (int kk = 0; kk < 8; kk += 2) {
                uint32_t b[4];
                ldsm_x4(b, Ks + (8u * pb + mr) * ROWB + 2u * (16u * (kk + (mi >> 1)) + 8u * (mi & 1u)));
                mma_f16_16816(sc[pb], qa[kk], b[0], b[1]);
                mma_f16_16816(sl[pb], qb[kk], b[0], b[1]);
                mma_f16_16816(sc[pb], qa[kk + 1], b[2], b[3]);
                mma_f16_16816(sl[pb], qb[kk + 1], b[2], b[3]);
            }
        }
#pragma unroll
        for (int pb = 0; pb < 2; ++pb)
#pragma unroll
            for (int c = 0; c < 4; ++c) sc[pb][c] += sl[pb][c];
        // causal mask and online softmax; element c of block pb: row g + 8(c >> 1), position 8pb + 2t + (c & 1)
        const uint32_t p0 = tile * PT;
#pragma unroll
        for (int pb = 0; pb < 2; ++pb)
#pragma unroll
            for (int c = 0; c < 4; ++c)
                if (p0 + 8u * pb + 2u * t + (c & 1) > lim[c >> 1]) sc[pb][c] = -INFINITY;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float mx = fmaxf(fmaxf(sc[0][2 * h], sc[0][2 * h + 1]), fmaxf(sc[1][2 * h], sc[1][2 * h + 1]));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            const float mn = fmaxf(m[h], mx);
            const float alpha = __expf(m[h] - mn);
            m[h] = mn;
            float ps = 0.f;
#pragma unroll
            for (int pb = 0; pb < 2; ++pb)
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    sc[pb][2 * h + c] = __expf(sc[pb][2 * h + c] - mn);
                    ps += sc[pb][2 * h + c];
                }
            ps += __shfl_xor_sync(0xffffffffu, ps, 1);
            ps += __shfl_xor_sync(0xffffffffu, ps, 2);
            l[h] = fmaf(l[h], alpha, ps);
#pragma unroll
            for (int nt = 0; nt < 16; ++nt) o[nt][2 * h] *= alpha, o[nt][2 * h + 1] *= alpha;
        }
        // O += P V with P (16 rows x 16 positions) from the S fragments
        const uint32_t pa[4] = {pack_f16(sc[0][0], sc[0][1]), pack_f16(sc[0][2], sc[0][3]),
                                pack_f16(sc[1][0], sc[1][1]), pack_f16(sc[1][2], sc[1][3])};
#pragma unroll
        for (int nt = 0; nt < 16; nt += 2) {
            uint32_t v[4];
            ldsm_x4_trans(v, Vs + (8u * (mi & 1u) + mr) * ROWB + 2u * (8u * (nt + (mi >> 1))));
            mma_f16_16816(o[nt], pa, v[0], v[1]);
            mma_f16_16816(o[nt + 1], pa, v[2], v[3]);
        }
        __syncwarp();  // this buffer is refilled two tiles later
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        if (!valid[h]) continue;
        uint16_t* dst = out + (uint64_t)qrow[h] * hdim + (kvh * GQ + head[h]) * D + 2u * t;
#pragma unroll
        for (int nt = 0; nt < 16; ++nt) {
            const uint32_t lo = f2bf(o[nt][2 * h] / l[h]), hi = f2bf(o[nt][2 * h + 1] / l[h]);
            *reinterpret_cast<uint32_t*>(dst + 8u * nt) = lo | (hi << 16);
        }
    }
}

__device__ __forceinline__ uint16_t silu_mul_bf16(float a, float u) { return f2bf((a / (1.0f + expf(-a))) * u); }

// Four elements per thread and step (float4 loads, one 8-byte store) when n % 4 == 0
// and the pointers allow it; otherwise one element at a time.  Same expression per element.
__global__ void silu_mul_rows_bf16_kernel(const float* __restrict__ g, const float* __restrict__ u, uint64_t n,
                                          uint16_t* __restrict__ out) {
    pdl_wait();  // inputs come from the preceding kernels
    const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x, stride = (uint64_t)gridDim.x * blockDim.x;
    const bool vec = (n % 4u) == 0u && ((reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(u)) & 15u) == 0u &&
                     (reinterpret_cast<uintptr_t>(out) & 7u) == 0u;
    if (vec) {
        const float4* g4 = reinterpret_cast<const float4*>(g);
        const float4* u4 = reinterpret_cast<const float4*>(u);
        uint2* o4 = reinterpret_cast<uint2*>(out);
        for (uint64_t i = tid; i < n / 4u; i += stride) {
            const float4 a = g4[i], b = u4[i];
            o4[i] = make_uint2((uint32_t)silu_mul_bf16(a.x, b.x) | ((uint32_t)silu_mul_bf16(a.y, b.y) << 16),
                               (uint32_t)silu_mul_bf16(a.z, b.z) | ((uint32_t)silu_mul_bf16(a.w, b.w) << 16));
        }
        return;
    }
    for (uint64_t i = tid; i < n; i += stride) out[i] = silu_mul_bf16(g[i], u[i]);
}

// After a batched prefill of positions 0 .. n_prompt-2: the decode graph
// continues with the last prompt token at its position.
__global__ void prefill_done_kernel(GreedyState* st, const uint32_t* __restrict__ prompt, uint32_t n_prompt) {
    pdl_wait();  // the prefill's last kernels may still be writing the cache
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
                             cudaStream_t stream, bool fp16, uint16_t* out_lo) {
    if (rows == 0) return ARC_OK;
    if (!x || !gamma || !out || h == 0) return set_error(ARC_E_INVALID_ARGUMENT, "rmsnorm rows: null pointer or h 0");
    const cudaError_t e =
        fp16 ? launch_kernel(rmsnorm_rows_bf16_kernel<true>, dim3(rows), dim3(256), 0, stream, x, gamma, eps, h, out,
                             out_lo, dev_error_word())
             : launch_kernel(rmsnorm_rows_bf16_kernel<false>, dim3(rows), dim3(256), 0, stream, x, gamma, eps, h, out,
                             static_cast<uint16_t*>(nullptr), dev_error_word());
    return launch_checked(e, "rmsnorm rows launch");
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
    if (((reinterpret_cast<uintptr_t>(kc) | reinterpret_cast<uintptr_t>(vc)) & 15u) ||
        (reinterpret_cast<uintptr_t>(q) & 7u) || (reinterpret_cast<uintptr_t>(out) & 3u))
        return set_error(ARC_E_ALIGNMENT, "attention prefill: caches 16-byte, q 8-byte, out 4-byte aligned");
    const uint32_t gq = s.q_heads / s.kv_heads;
    if (gq * s.kv_heads != s.q_heads) return set_error(ARC_E_UNSUPPORTED_SHAPE, "attention: q_heads % kv_heads");
    // two warps per CTA, each 16 / (q heads per KV head, 7 -> 8) query rows
    const uint32_t rq = 16u / (gq == 7u ? 8u : gq);
    const dim3 grid((rows + 2u * rq - 1u) / (2u * rq), s.kv_heads);
    unsigned int* err = dev_error_word();
    cudaError_t e;
    switch (gq) {
        case 1: e = launch_kernel(attention_prefill_kernel<1>, grid, dim3(64), 0, stream, q, kc, vc, pos0, rows, s, out, err); break;
        case 2: e = launch_kernel(attention_prefill_kernel<2>, grid, dim3(64), 0, stream, q, kc, vc, pos0, rows, s, out, err); break;
        case 4: e = launch_kernel(attention_prefill_kernel<4>, grid, dim3(64), 0, stream, q, kc, vc, pos0, rows, s, out, err); break;
        case 7: e = launch_kernel(attention_prefill_kernel<7>, grid, dim3(64), 0, stream, q, kc, vc, pos0, rows, s, out, err); break;
        case 8: e = launch_kernel(attention_prefill_kernel<8>, grid, dim3(64), 0, stream, q, kc, vc, pos0, rows, s, out, err); break;
        default: return set_error(ARC_E_UNSUPPORTED_SHAPE, "attention: q heads per kv head must be 1, 2, 4, 7 or 8");
    }
    return launch_checked(e, "attention prefill launch");
}

int launch_silu_mul_rows_bf16(const float* g, const float* u, uint64_t n, uint16_t* out, cudaStream_t stream) {
    if (n == 0) return ARC_OK;
    const uint32_t blocks = (uint32_t)std::min<uint64_t>((n / 4u + 255) / 256 + 1u, 148u * 16u);
    return launch_checked(launch_kernel(silu_mul_rows_bf16_kernel, dim3(blocks), dim3(256), 0, stream, g, u, n, out),
                          "silu mul launch");
}

}  // namespace arc
