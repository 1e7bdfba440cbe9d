// M=1 dequant-matvec over GGUF-packed Q4_K / Q6_K weights, B200 (sm_100a).
//
// Replaces the reference's decode matvec shaders
//   shaders/p7_q4k_gemm_2d.comp, shaders/p7_q6k_gemm_2d.comp (1 thread/row),
//   shaders/sa1_q4k_subgroup_splitk.comp (32-lane split-K, "I002"),
//   shaders/p8q1_lmhead_q6k_segmented_chunk.comp (LM head chunks),
// plus the elementwise passes the runtime issues around them
//   shaders/p7_rmsnorm_seq.comp (fused into the x staging),
//   shaders/p7_add.comp (fused as a residual epilogue),
//   shaders/p7_swiglu.comp (fused into the dual gate/up form)
// (call sites: src/arcllm_v1_runtime.cpp:378-418).
//
// Design (HBM-bound streaming, no tensor cores):
//   * rows are processed in groups of G rows; a group's bytes G*row_bytes are
//     contiguous and 16-byte aligned, so ONE producer thread per CTA streams
//     whole groups into a ring of shared-memory stages with 1-D TMA bulk
//     copies (cp.async.bulk + mbarrier complete_tx, L2 evict_first).  Q6_K's
//     210-byte super-blocks are not 16-byte aligned individually; groups of
//     8/gcd(nb,8) rows are, which is what makes the bulk copy legal;
//   * 8 consumer warps split K: each consumer thread owns fixed positions
//     (a 32-weight Q4_K chunk or a 16-weight Q6_K l-quad) and applies them to
//     every row of the stage, so each x value read from shared memory is
//     reused G times;
//   * codes are turned into floats without integer->float conversions: a
//     byte q is placed into the mantissa of 0.5f (PRMT), giving exactly
//     0.5 + q/256; sum(q*x) = 256*sum(f*x) - 128*sum(x);
//   * per-row partial sums are folded with a multi-value butterfly (one
//     shuffle per value per step) and summed across warps in shared memory;
//     the epilogue adds bias / residual or applies silu(g)*u.
#include <algorithm>
#include <cstdio>

#include "arcllm_cuda_internal.h"
#include "common.cuh"

namespace arc {

namespace {

constexpr int kNW = 8;                 // consumer warps
constexpr int kNT = kNW * 32;          // consumer threads
constexpr int kThreads = kNT + 32;     // + one producer warp
constexpr int kMaxStages = 8;
constexpr uint32_t kStagePad = 16;     // slack after each stage for unaligned 32-bit reads

struct MvParams {
    const uint8_t* w0;
    const uint8_t* w1;  // second matrix of the dual (gate/up) form
    const float* x;
    const float* gamma;  // fused RMSNorm weight (nullable)
    float eps;
    const float* bias;      // nullable
    const float* residual;  // nullable
    float* y;
    unsigned int* err;  // device error word
    uint32_t rows, k, nb, rb;
    uint32_t G;          // rows per group (<= GMAX)
    uint32_t n_groups;
    uint32_t stages;
    uint32_t stage_smem;  // bytes of one stage in smem (both matrices + pad)
    uint32_t x_floats;    // padded x length in smem
};

// x lives in shared memory with 4 floats of padding every 64, so the eight
// lanes of a quarter-warp that read x runs 64 floats apart hit distinct banks.
__device__ __forceinline__ uint32_t xpad(uint32_t e) { return e + ((e >> 6) << 2); }

__host__ __device__ constexpr uint32_t xpad_len(uint32_t k) { return k + (k >> 4); }

// 0.5 + byte/256 as fp32 (byte c of v moved into bits 16..23 under 0x3F).
__device__ __forceinline__ float q2f(uint32_t v, uint32_t c) {
    return __uint_as_float(__byte_perm(v, 0x3F000000u, 0x7044u | (c << 8)));
}

__device__ __forceinline__ float dot4(uint32_t v, const float4& xv, float acc) {
    acc = fmaf(q2f(v, 0), xv.x, acc);
    acc = fmaf(q2f(v, 1), xv.y, acc);
    acc = fmaf(q2f(v, 2), xv.z, acc);
    acc = fmaf(q2f(v, 3), xv.w, acc);
    return acc;
}

__device__ __forceinline__ float hsum4(const float4& v) { return (v.x + v.y) + (v.z + v.w); }

// 32-bit little-endian read at an even (possibly not 4-aligned) smem offset.
__device__ __forceinline__ uint32_t lds_u32_even(const uint8_t* base, uint32_t off) {
    const uint32_t* p = reinterpret_cast<const uint32_t*>(base + (off & ~3u));
    return __funnelshift_r(p[0], p[1], (off & 3u) * 8u);
}

// Fold N per-row partial sums over the warp: afterwards lane L holds the full
// sum of value index (L >> (5 - log2 N)).  One shuffle per value per step.
template <int N>
__device__ __forceinline__ float warp_fold(float (&v)[N], uint32_t lane) {
    static_assert(N >= 1 && N <= 32 && (N & (N - 1)) == 0, "N must be a power of two <= 32");
    int n = N;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        if (n > 1) {
            const int h = n >> 1;
            const bool upper = (lane & o) != 0;
#pragma unroll
            for (int i = 0; i < N / 2; ++i) {
                if (i < h) {
                    const float send = upper ? v[i] : v[i + h];
                    const float keep = upper ? v[i + h] : v[i];
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
                }
            }
            n = h;
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
        }
    }
    return v[0];
}

template <int GMAX, bool DUAL>
struct Acc {
    float v[DUAL ? 2 * GMAX : GMAX];
};

// ---- per-format decode of one owned position over all rows of a stage ----
template <int GMAX, bool DUAL>
__device__ __forceinline__ void q4k_position(const uint8_t* st, uint32_t stage_mat_off, uint32_t rb,
                                             uint32_t rows_g, uint32_t p, const float* xs,
                                             Acc<GMAX, DUAL>& acc) {
    const uint32_t b = p >> 3, m = p & 7u, g = m >> 1, hs = m & 1u;
    const uint32_t xe = b * 256u + g * 64u + hs * 16u;
    float4 xl[4], xh[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        xl[i] = *reinterpret_cast<const float4*>(xs + xpad(xe + 4u * i));
        xh[i] = *reinterpret_cast<const float4*>(xs + xpad(xe + 32u + 4u * i));
    }
    const float sxl = (hsum4(xl[0]) + hsum4(xl[1])) + (hsum4(xl[2]) + hsum4(xl[3]));
    const float sxh = (hsum4(xh[0]) + hsum4(xh[1])) + (hsum4(xh[2]) + hsum4(xh[3]));
    const uint32_t sh = (g & 1u) * 16u;  // byte offset of sub-block 2g within its 4-byte word group
    const bool hi_sb = g >= 2u;
#pragma unroll
    for (int mat = 0; mat < (DUAL ? 2 : 1); ++mat) {
#pragma unroll
        for (int r = 0; r < GMAX; ++r) {
            if (r < (int)rows_g) {
                const uint8_t* blk = st + mat * stage_mat_off + r * rb + b * 144u;
                const uint4 hd = *reinterpret_cast<const uint4*>(blk);
                const uint4 qv = *reinterpret_cast<const uint4*>(blk + 16u + m * 16u);
                const float d = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xffffu)));
                const float dmin = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
                // scale/min bytes of sub-blocks j0 = 2g and j1 = 2g+1
                const uint32_t A = hd.y >> sh, B = hd.z >> sh, Cc = hd.w >> sh;
                uint32_t sc0, mn0, sc1, mn1;
                if (!hi_sb) {
                    sc0 = A & 63u;
                    mn0 = B & 63u;
                    sc1 = (A >> 8) & 63u;
                    mn1 = (B >> 8) & 63u;
                } else {
                    sc0 = (Cc & 15u) | ((A >> 2) & 0x30u);
                    mn0 = ((Cc >> 4) & 15u) | ((B >> 2) & 0x30u);
                    sc1 = ((Cc >> 8) & 15u) | ((A >> 10) & 0x30u);
                    mn1 = ((Cc >> 12) & 15u) | ((B >> 10) & 0x30u);
                }
                float sl = 0.f, shh = 0.f;
                const uint32_t q[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    sl = dot4(q[i] & 0x0F0F0F0Fu, xl[i], sl);
                    shh = dot4((q[i] >> 4) & 0x0F0F0F0Fu, xh[i], shh);
                }
                const float sum_lo = fmaf(256.f, sl, -128.f * sxl);
                const float sum_hi = fmaf(256.f, shh, -128.f * sxh);
                const float t = fmaf((float)sc0, sum_lo, (float)sc1 * sum_hi);
                const float u = fmaf((float)mn0, sxl, (float)mn1 * sxh);
                acc.v[mat * GMAX + r] += fmaf(d, t, -dmin * u);
            }
        }
    }
}

template <int GMAX, bool DUAL>
__device__ __forceinline__ void q6k_position(const uint8_t* st, uint32_t stage_mat_off, uint32_t rb,
                                             uint32_t rows_g, uint32_t p, const float* xs,
                                             Acc<GMAX, DUAL>& acc) {
    const uint32_t b = p >> 4, h = (p >> 3) & 1u, j8 = p & 7u, l0 = 4u * j8;
    const uint32_t xe = b * 256u + h * 128u + l0;
    float4 xq[4];
    float X[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        xq[q] = *reinterpret_cast<const float4*>(xs + xpad(xe + 32u * q));
        X[q] = hsum4(xq[q]);
    }
#pragma unroll
    for (int mat = 0; mat < (DUAL ? 2 : 1); ++mat) {
#pragma unroll
        for (int r = 0; r < GMAX; ++r) {
            if (r < (int)rows_g) {
                const uint32_t blk = mat * stage_mat_off + r * rb + b * 210u;
                const uint32_t ql0 = lds_u32_even(st, blk + h * 64u + l0);
                const uint32_t ql1 = lds_u32_even(st, blk + h * 64u + 32u + l0);
                const uint32_t qh = lds_u32_even(st, blk + 128u + h * 32u + l0);
                const int8_t* scp = reinterpret_cast<const int8_t*>(st + blk + 192u + h * 8u + (j8 >> 2));
                const float d = __half2float(
                    __ushort_as_half(*reinterpret_cast<const unsigned short*>(st + blk + 208u)));
                const uint32_t v0 = (ql0 & 0x0F0F0F0Fu) | ((qh << 4) & 0x30303030u);
                const uint32_t v1 = (ql1 & 0x0F0F0F0Fu) | ((qh << 2) & 0x30303030u);
                const uint32_t v2 = ((ql0 >> 4) & 0x0F0F0F0Fu) | (qh & 0x30303030u);
                const uint32_t v3 = ((ql1 >> 4) & 0x0F0F0F0Fu) | ((qh >> 2) & 0x30303030u);
                const float s0 = fmaf(256.f, dot4(v0, xq[0], 0.f), -160.f * X[0]);
                const float s1 = fmaf(256.f, dot4(v1, xq[1], 0.f), -160.f * X[1]);
                const float s2 = fmaf(256.f, dot4(v2, xq[2], 0.f), -160.f * X[2]);
                const float s3 = fmaf(256.f, dot4(v3, xq[3], 0.f), -160.f * X[3]);
                float t = (float)scp[0] * s0;
                t = fmaf((float)scp[2], s1, t);
                t = fmaf((float)scp[4], s2, t);
                t = fmaf((float)scp[6], s3, t);
                acc.v[mat * GMAX + r] = fmaf(d, t, acc.v[mat * GMAX + r]);
            }
        }
    }
}

template <int FMT, int GMAX, bool DUAL>
__global__ void __launch_bounds__(kThreads, 1) matvec_stream_kernel(const MvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kMaxStages;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kMaxStages);
    double* red_d = reinterpret_cast<double*>(smem + 2 * kMaxStages * 8 + 16);  // kNW doubles
    constexpr int NV = DUAL ? 2 * GMAX : GMAX;
    float* red = reinterpret_cast<float*>(red_d + kNW);                            // [2][kNW][NV]
    float* xs = red + 2 * kNW * NV;
    xs = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(xs) + 15) & ~uintptr_t(15));
    uint8_t* stages = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(xs + p.x_floats) + 127) & ~uintptr_t(127));

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    const uint32_t S = p.stages;
    const uint32_t mat_off = p.G * p.rb;  // offset of the second matrix inside a stage

    if (tid == kNT) {
        for (uint32_t s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kNW);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kNW) {
        // ---------------- producer warp ----------------
        const uint64_t pol = l2_evict_first_policy();
        uint32_t it = 0;
        for (uint32_t grp = blockIdx.x; grp < p.n_groups; grp += gridDim.x, ++it) {
            const uint32_t s = it % S;
            if (it >= S) {
                bool ok = true;
                if (lane == 0) ok = mbar_wait(&empty[s], ((it / S) - 1u) & 1u, p.err);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) {
                    if (lane == 0) *abort_flag = 1;
                    break;
                }
            }
            const uint32_t rows_g = min(p.G, p.rows - grp * p.G);
            const uint32_t bytes = rows_g * p.rb;
            const uint32_t bulk = bytes & ~15u;
            uint8_t* dst = stages + s * p.stage_smem;
            const uint64_t goff = (uint64_t)grp * p.G * p.rb;
            if (bytes != bulk) {  // ragged final group: copy the last <16 bytes by hand
                for (uint32_t i = bulk + lane; i < bytes; i += 32) {
                    dst[i] = p.w0[goff + i];
                    if (DUAL) dst[mat_off + i] = p.w1[goff + i];
                }
                __syncwarp();
            }
            if (lane == 0) {
                mbar_arrive_expect_tx(&full[s], bulk * (DUAL ? 2u : 1u));
                for (uint32_t o = 0; o < bulk; o += 32768u) {
                    const uint32_t n = min(32768u, bulk - o);
                    bulk_g2s(dst + o, p.w0 + goff + o, n, &full[s], pol);
                    if (DUAL) bulk_g2s(dst + mat_off + o, p.w1 + goff + o, n, &full[s], pol);
                }
            }
        }
        // drain: make sure no bulk copy is still landing in this CTA's smem
        if (lane == 0 && *abort_flag) {
            const uint32_t first = it > S ? it - S : 0;
            for (uint32_t j = first; j < it; ++j) mbar_wait(&full[j % S], (j / S) & 1u, p.err);
        }
        return;
    }

    // ---------------- consumer warps ----------------
    // stage x (optionally RMS-normalised, src/p8c_segmented_access_correctness.cpp:958-969)
    float inv = 1.0f;
    if (p.gamma) {
        double ss = 0.0;
        for (uint32_t i = tid; i < p.k; i += kNT) {
            const double v = (double)p.x[i];
            ss += v * v;
        }
        ss = warp_sum_d(ss);
        if (lane == 0) red_d[warp] = ss;
        named_bar_sync(1, kNT);
        double tot = 0.0;
#pragma unroll
        for (int w = 0; w < kNW; ++w) tot += red_d[w];
        inv = 1.0f / sqrtf((float)(tot / (double)p.k) + p.eps);
    }
    for (uint32_t i = tid; i < p.k; i += kNT) {
        float v = p.x[i];
        if (p.gamma) v = (v * inv) * p.gamma[i];
        xs[xpad(i)] = v;
    }
    named_bar_sync(1, kNT);

    const uint32_t P = (FMT == 12) ? p.nb * 8u : p.nb * 16u;
    uint32_t it = 0, buf = 0;
    for (uint32_t grp = blockIdx.x; grp < p.n_groups; grp += gridDim.x, ++it, buf ^= 1u) {
        const uint32_t s = it % S;
        const bool ok = mbar_wait(&full[s], (it / S) & 1u, p.err);
        if (!ok) *abort_flag = 1;
        const uint32_t rows_g = min(p.G, p.rows - grp * p.G);
        const uint8_t* st = stages + s * p.stage_smem;
        Acc<GMAX, DUAL> acc;
#pragma unroll
        for (int i = 0; i < NV; ++i) acc.v[i] = 0.f;
        if (ok) {
            for (uint32_t pos = tid; pos < P; pos += kNT) {
                if (FMT == 12)
                    q4k_position<GMAX, DUAL>(st, mat_off, p.rb, rows_g, pos, xs, acc);
                else
                    q6k_position<GMAX, DUAL>(st, mat_off, p.rb, rows_g, pos, xs, acc);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        const float v = warp_fold<NV>(acc.v, lane);
        constexpr uint32_t kShift = 5u - (NV == 1 ? 0 : NV == 2 ? 1 : NV == 4 ? 2 : NV == 8 ? 3 : NV == 16 ? 4 : 5);
        if ((lane & ((1u << kShift) - 1u)) == 0u) red[(buf * kNW + warp) * NV + (lane >> kShift)] = v;
        named_bar_sync(1, kNT);
        if (*abort_flag) break;
        if (tid < rows_g) {
            const uint32_t row = grp * p.G + tid;
            float a = 0.f;
#pragma unroll
            for (int w = 0; w < kNW; ++w) a += red[(buf * kNW + w) * NV + tid];
            if (DUAL) {
                float u = 0.f;
#pragma unroll
                for (int w = 0; w < kNW; ++w) u += red[(buf * kNW + w) * NV + GMAX + tid];
                // src/p8c_segmented_access_correctness.cpp:1064-1073 (silu(g)*u)
                p.y[row] = (a / (1.0f + expf(-a))) * u;
            } else {
                if (p.bias) a += p.bias[row];
                if (p.residual) a = p.residual[row] + a;
                p.y[row] = a;
            }
        }
    }
}

struct DevInfo {
    int sms = 0;
    int max_smem = 0;
};

DevInfo dev_info() {
    static DevInfo cache[64];
    int dev = 0;
    cudaGetDevice(&dev);
    DevInfo& d = cache[dev & 63];
    if (d.sms == 0) {
        cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
        cudaDeviceGetAttribute(&d.max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    }
    return d;
}

template <int FMT, int GMAX, bool DUAL>
cudaError_t launch_t(const MvParams& p, uint32_t smem, uint32_t grid, cudaStream_t stream) {
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_set[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(matvec_stream_kernel<FMT, GMAX, DUAL>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        attr_set[dev & 63] = true;
    }
    matvec_stream_kernel<FMT, GMAX, DUAL><<<grid, kThreads, smem, stream>>>(p);
    return cudaGetLastError();
}

uint32_t gcd_u(uint32_t a, uint32_t b) {
    while (b) {
        uint32_t t = a % b;
        a = b;
        b = t;
    }
    return a;
}

}  // namespace

int matvec_plan(int fmt, bool dual, uint32_t rows, uint32_t k, MatvecPlan* out) {
    if (fmt != 12 && fmt != 14) return set_error(ARC_E_INVALID_ARGUMENT, "matvec: format must be Q4_K (12) or Q6_K (14)");
    if (dual && fmt != 12) return set_error(ARC_E_UNSUPPORTED_SHAPE, "matvec: the dual gate/up form is Q4_K only");
    if (rows == 0 || k == 0 || (k % 256u) != 0u)
        return set_error(ARC_E_INVALID_ARGUMENT, "matvec: rows must be >= 1 and k a non-zero multiple of 256");
    if (k > 32768u) return set_error(ARC_E_UNSUPPORTED_SHAPE, "matvec: k > 32768 is not supported");
    const uint32_t nb = k / 256u;
    const uint32_t rb = nb * (fmt == 12 ? 144u : 210u);
    const uint32_t gmin = fmt == 12 ? 1u : 8u / gcd_u(nb, 8u);
    const uint32_t mats = dual ? 2u : 1u;
    const uint32_t target = 32u * 1024u;
    uint32_t gmax_t = dual ? 8u : 16u;
    uint32_t G = gmin;
    while (G + gmin <= gmax_t && (G + gmin) * rb * mats <= target) G += gmin;
    if (G > gmax_t) return set_error(ARC_E_UNSUPPORTED_SHAPE, "matvec: row group does not fit");
    const uint32_t GM = G <= 4 ? 4u : (G <= 8 ? 8u : 16u);
    const uint32_t NV = GM * mats;
    const uint32_t stage_smem = ((G * rb * mats + kStagePad) + 127u) & ~127u;
    const uint32_t x_floats = xpad_len(k);
    const uint32_t fixed = 2 * kMaxStages * 8 + 16 + kNW * 8 + 2 * kNW * NV * 4 + 16 + x_floats * 4 + 128;
    const DevInfo di = dev_info();
    const uint32_t smem_cap = di.max_smem > 0 ? (uint32_t)di.max_smem : 227u * 1024u;
    // aim for two CTAs per SM, fall back to one
    uint32_t ctas_per_sm = 2;
    uint32_t budget = smem_cap / 2u - 1024u;
    int64_t S = ((int64_t)budget - fixed) / stage_smem;
    if (S < 3) {
        ctas_per_sm = 1;
        budget = smem_cap - 1024u;
        S = ((int64_t)budget - fixed) / stage_smem;
    }
    if (S < 2) return set_error(ARC_E_UNSUPPORTED_SHAPE, "matvec: not enough shared memory for two stages");
    if (S > kMaxStages) S = kMaxStages;
    out->fmt = fmt;
    out->dual = dual;
    out->rows = rows;
    out->k = k;
    out->nb = nb;
    out->rb = rb;
    out->G = G;
    out->gmax = GM;
    out->n_groups = (rows + G - 1u) / G;
    out->stages = (uint32_t)S;
    out->stage_smem = stage_smem;
    out->x_floats = x_floats;
    out->smem = fixed + (uint32_t)S * stage_smem;
    const uint32_t sms = di.sms > 0 ? (uint32_t)di.sms : 148u;
    out->grid = std::min(out->n_groups, sms * ctas_per_sm);
    return ARC_OK;
}

int matvec_launch(const MatvecPlan& pl, const void* w0, const void* w1, const float* x, const float* gamma,
                  float eps, const float* bias, const float* residual, float* y, cudaStream_t stream) {
    if (!w0 || !x || !y || (pl.dual && !w1)) return set_error(ARC_E_INVALID_ARGUMENT, "matvec: null pointer");
    if ((reinterpret_cast<uintptr_t>(w0) & 15u) || (w1 && (reinterpret_cast<uintptr_t>(w1) & 15u)))
        return set_error(ARC_E_ALIGNMENT, "matvec: weight pointers must be 16-byte aligned");
    MvParams p{};
    p.w0 = static_cast<const uint8_t*>(w0);
    p.w1 = static_cast<const uint8_t*>(w1);
    p.x = x;
    p.gamma = gamma;
    p.eps = eps;
    p.bias = bias;
    p.residual = residual;
    p.y = y;
    p.err = dev_error_word();
    p.rows = pl.rows;
    p.k = pl.k;
    p.nb = pl.nb;
    p.rb = pl.rb;
    p.G = pl.G;
    p.n_groups = pl.n_groups;
    p.stages = pl.stages;
    p.stage_smem = pl.stage_smem;
    p.x_floats = pl.x_floats;
    cudaError_t e;
    if (pl.fmt == 12) {
        if (pl.dual) {
            e = pl.gmax == 4 ? launch_t<12, 4, true>(p, pl.smem, pl.grid, stream)
                             : launch_t<12, 8, true>(p, pl.smem, pl.grid, stream);
        } else {
            e = pl.gmax == 4   ? launch_t<12, 4, false>(p, pl.smem, pl.grid, stream)
                : pl.gmax == 8 ? launch_t<12, 8, false>(p, pl.smem, pl.grid, stream)
                               : launch_t<12, 16, false>(p, pl.smem, pl.grid, stream);
        }
    } else {
        e = pl.gmax == 4   ? launch_t<14, 4, false>(p, pl.smem, pl.grid, stream)
            : pl.gmax == 8 ? launch_t<14, 8, false>(p, pl.smem, pl.grid, stream)
                           : launch_t<14, 16, false>(p, pl.smem, pl.grid, stream);
    }
    if (e != cudaSuccess) return set_cuda_error(e, "matvec launch");
    return ARC_OK;
}

}  // namespace arc
