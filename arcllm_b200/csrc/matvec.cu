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
// Design (HBM streaming on CUDA cores, no tensor cores):
//   * rows are processed in groups of G rows; a group's bytes G*row_bytes are
//     contiguous and 16-byte aligned, so ONE producer thread per CTA streams
//     whole groups into a ring of shared-memory stages with 1-D TMA bulk
//     copies (cp.async.bulk + mbarrier complete_tx, L2 evict_first).  Q6_K's
//     210-byte super-blocks are not 16-byte aligned individually; groups of
//     8/gcd(nb,8) rows are, which is what makes the bulk copy legal;
//   * consumer warps split K into 32-weight units (a Q4_K 16-byte nibble chunk,
//     or a Q6_K run of 8 l-positions over its 4 quarters) -- 8 units per
//     super-block for both formats.  Each consumer thread owns fixed units and
//     applies them to every row of a stage, so x is read once per G rows; when
//     every thread owns at most one unit (K <= 4096) x stays in registers for
//     the whole kernel;
//   * codes become floats without int->float conversion: byte q is placed in
//     the mantissa of 0.5f with one PRMT, giving exactly 0.5 + q/256, and
//     sum(q*x) = 256*sum(f*x) - 128*sum(x).  The products run as packed
//     fma.rn.f32x2 (two fp32 FMAs per instruction);
//   * no CTA-wide barrier in the steady state: each warp folds its per-row
//     partials with a multi-value butterfly, stores them, and the LAST warp to
//     finish a stage (shared-memory counter) sums the warps' partials in fixed
//     order -- results are deterministic -- and runs the epilogue (bias,
//     residual, or silu(g)*u).
#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "arcllm_cuda_internal.h"
#include "common.cuh"
#include "matvec_common.cuh"

namespace arc {

namespace {

// x lives in shared memory with 4 floats of padding every 64 so that the
// eight lanes of a quarter-warp reading runs 64 floats apart hit distinct banks.
__device__ __forceinline__ uint32_t xpad(uint32_t e) { return e + ((e >> 6) << 2); }
__host__ __device__ constexpr uint32_t xpad_len(uint32_t k) { return k + (k >> 4) + 4; }

// 0.5 + (byte c of v)/256 as fp32 (the byte moved into bits 16..23 under 0x3F).
__device__ __forceinline__ float q2f(uint32_t v, uint32_t c) {
    return __uint_as_float(__byte_perm(v, 0x3F000000u, 0x7044u | (c << 8)));
}

// acc += (a.x*b.x, a.y*b.y) as one packed fma.rn.f32x2
__device__ __forceinline__ void ffma2(float2& acc, float ax, float ay, float bx, float by) {
    asm("{\n\t.reg .b64 a, b, c;\n\t"
        "mov.b64 a, {%2, %3};\n\t"
        "mov.b64 b, {%4, %5};\n\t"
        "mov.b64 c, {%0, %1};\n\t"
        "fma.rn.f32x2 c, a, b, c;\n\t"
        "mov.b64 {%0, %1}, c;\n\t}"
        : "+f"(acc.x), "+f"(acc.y)
        : "f"(ax), "f"(ay), "f"(bx), "f"(by));
}

// sum over the 4 bytes of v of (0.5 + byte/256) * x[i], accumulated in acc
__device__ __forceinline__ void dot4x2(uint32_t v, const float* x, float2& acc) {
    ffma2(acc, q2f(v, 0), q2f(v, 1), x[0], x[1]);
    ffma2(acc, q2f(v, 2), q2f(v, 3), x[2], x[3]);
}

// 64-bit little-endian read at an even (possibly not 4-aligned) smem byte offset
__device__ __forceinline__ void lds_u64_even(const uint8_t* base, uint32_t off, uint32_t& lo, uint32_t& hi) {
    const uint32_t* p = reinterpret_cast<const uint32_t*>(base + (off & ~3u));
    const uint32_t sh = (off & 3u) * 8u;
    const uint32_t w0 = p[0], w1 = p[1], w2 = p[2];
    lo = __funnelshift_r(w0, w1, sh);
    hi = __funnelshift_r(w1, w2, sh);
}

// ---------------------------------------------------------------------------
// x values of one 32-weight unit (registers)
//   Q4_K unit (b, m): lo run  x[b*256 + (m>>1)*64 + (m&1)*16 + 0..15]
//                     hi run  the same + 32           (16 + 16 floats)
//   Q6_K unit (b, h, j): quarter q run x[b*256 + h*128 + 32q + 8j + 0..7]
// ---------------------------------------------------------------------------
struct UnitX {
    float v[32];
    float s[4];  // Q4: s[0]=sum lo, s[1]=sum hi;  Q6: per-quarter sums
};

template <int FMT>
__device__ __forceinline__ void load_unit_x(const float* xs, uint32_t u, UnitX& X) {
    const uint32_t b = u >> 3, m = u & 7u;
    if (FMT == 12) {
        const uint32_t xe = b * 256u + (m >> 1) * 64u + (m & 1u) * 16u;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float4 a = *reinterpret_cast<const float4*>(xs + xpad(xe + 4u * i));
            const float4 c = *reinterpret_cast<const float4*>(xs + xpad(xe + 32u + 4u * i));
            X.v[4 * i + 0] = a.x, X.v[4 * i + 1] = a.y, X.v[4 * i + 2] = a.z, X.v[4 * i + 3] = a.w;
            X.v[16 + 4 * i + 0] = c.x, X.v[16 + 4 * i + 1] = c.y, X.v[16 + 4 * i + 2] = c.z,
                             X.v[16 + 4 * i + 3] = c.w;
        }
        float a = 0.f, c = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) a += X.v[i], c += X.v[16 + i];
        X.s[0] = a, X.s[1] = c, X.s[2] = 0.f, X.s[3] = 0.f;
    } else {
        const uint32_t h = m >> 2, j = m & 3u;
        const uint32_t xe = b * 256u + h * 128u + 8u * j;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float4 a = *reinterpret_cast<const float4*>(xs + xpad(xe + 32u * q));
            const float4 c = *reinterpret_cast<const float4*>(xs + xpad(xe + 32u * q + 4u));
            X.v[8 * q + 0] = a.x, X.v[8 * q + 1] = a.y, X.v[8 * q + 2] = a.z, X.v[8 * q + 3] = a.w;
            X.v[8 * q + 4] = c.x, X.v[8 * q + 5] = c.y, X.v[8 * q + 6] = c.z, X.v[8 * q + 7] = c.w;
            float t = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) t += X.v[8 * q + i];
            X.s[q] = t;
        }
    }
}

// contribution of unit u of block-row `blk` (byte offset into the stage) for one row
__device__ __forceinline__ float q4k_unit(const uint8_t* st, uint32_t blk, uint32_t m, const UnitX& X) {
    const uint4 hd = *reinterpret_cast<const uint4*>(st + blk);
    const uint4 qv = *reinterpret_cast<const uint4*>(st + blk + 16u + m * 16u);
    const uint32_t g = m >> 1, sh = (g & 1u) * 16u;
    const float d = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xffffu)));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
    const uint32_t A = hd.y >> sh, B = hd.z >> sh, Cc = hd.w >> sh;
    uint32_t sc0, mn0, sc1, mn1;
    if (g < 2u) {
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
    // four independent accumulation chains (lo/hi nibbles x even/odd words)
    float2 al[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
    float2 ah[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
    const uint32_t q[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        dot4x2(q[i] & 0x0F0F0F0Fu, &X.v[4 * i], al[i & 1]);
        dot4x2((q[i] >> 4) & 0x0F0F0F0Fu, &X.v[16 + 4 * i], ah[i & 1]);
    }
    const float sum_lo = fmaf(256.f, (al[0].x + al[0].y) + (al[1].x + al[1].y), -128.f * X.s[0]);
    const float sum_hi = fmaf(256.f, (ah[0].x + ah[0].y) + (ah[1].x + ah[1].y), -128.f * X.s[1]);
    const float t = fmaf((float)sc0, sum_lo, (float)sc1 * sum_hi);
    const float u = fmaf((float)mn0, X.s[0], (float)mn1 * X.s[1]);
    return fmaf(d, t, -dmin * u);
}

__device__ __forceinline__ float q6k_unit(const uint8_t* st, uint32_t blk, uint32_t m, const UnitX& X) {
    const uint32_t h = m >> 2, l0 = 8u * (m & 3u);
    uint32_t a0, a1, b0, b1, h0, h1;
    lds_u64_even(st, blk + h * 64u + l0, a0, a1);        // ql[l0..l0+7]      (quarters 0 / 2)
    lds_u64_even(st, blk + h * 64u + 32u + l0, b0, b1);  // ql[32+l0..]       (quarters 1 / 3)
    lds_u64_even(st, blk + 128u + h * 32u + l0, h0, h1); // qh[l0..l0+7]
    const int8_t* scp = reinterpret_cast<const int8_t*>(st + blk + 192u + h * 8u + (l0 >> 4));
    const float d = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(st + blk + 208u)));
    float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
    const uint32_t qa[2] = {a0, a1}, qb[2] = {b0, b1}, qh[2] = {h0, h1};
#pragma unroll
    for (int w = 0; w < 2; ++w) {
        const uint32_t v0 = (qa[w] & 0x0F0F0F0Fu) | ((qh[w] << 4) & 0x30303030u);
        const uint32_t v1 = (qb[w] & 0x0F0F0F0Fu) | ((qh[w] << 2) & 0x30303030u);
        const uint32_t v2 = ((qa[w] >> 4) & 0x0F0F0F0Fu) | (qh[w] & 0x30303030u);
        const uint32_t v3 = ((qb[w] >> 4) & 0x0F0F0F0Fu) | ((qh[w] >> 2) & 0x30303030u);
        dot4x2(v0, &X.v[0 + 4 * w], acc[0]);
        dot4x2(v1, &X.v[8 + 4 * w], acc[1]);
        dot4x2(v2, &X.v[16 + 4 * w], acc[2]);
        dot4x2(v3, &X.v[24 + 4 * w], acc[3]);
    }
    // sum((q-32)*x) = 256*sum(f*x) - 128*sum(x) - 32*sum(x)
    float t = (float)scp[0] * fmaf(256.f, acc[0].x + acc[0].y, -160.f * X.s[0]);
    t = fmaf((float)scp[2], fmaf(256.f, acc[1].x + acc[1].y, -160.f * X.s[1]), t);
    t = fmaf((float)scp[4], fmaf(256.f, acc[2].x + acc[2].y, -160.f * X.s[2]), t);
    t = fmaf((float)scp[6], fmaf(256.f, acc[3].x + acc[3].y, -160.f * X.s[3]), t);
    return d * t;
}

template <int FMT, int G, bool DUAL>
__device__ __forceinline__ void apply_unit(const uint8_t* st, uint32_t mat_off, uint32_t rb, uint32_t rows_g,
                                           uint32_t u, const UnitX& X, float (&acc)[DUAL ? 2 * G : G]) {
    const uint32_t b = u >> 3, m = u & 7u;
    const uint32_t b0 = b * (FMT == 12 ? 144u : 210u);
    if (rows_g == (uint32_t)G) {  // full group: no predication, rows interleave freely
#pragma unroll
        for (int mat = 0; mat < (DUAL ? 2 : 1); ++mat) {
#pragma unroll
            for (int r = 0; r < G; ++r) {
                const uint32_t blk = mat * mat_off + r * rb + b0;
                acc[mat * G + r] += (FMT == 12) ? q4k_unit(st, blk, m, X) : q6k_unit(st, blk, m, X);
            }
        }
    } else {
#pragma unroll
        for (int mat = 0; mat < (DUAL ? 2 : 1); ++mat) {
#pragma unroll
            for (int r = 0; r < G; ++r) {
                if (r < (int)rows_g) {
                    const uint32_t blk = mat * mat_off + r * rb + b0;
                    acc[mat * G + r] += (FMT == 12) ? q4k_unit(st, blk, m, X) : q6k_unit(st, blk, m, X);
                }
            }
        }
    }
}

// x values of unit u straight from global memory (XREG mode): xn = x, or
// (x * inv) * gamma with the same rounding as the shared-memory staging.
template <int FMT>
__device__ __forceinline__ void load_unit_x_global(const float* x, const float* gamma, float inv, uint32_t u,
                                                   UnitX& X) {
    const uint32_t b = u >> 3, m = u & 7u;
    uint32_t base[4];
    int runs, len;
    if (FMT == 12) {
        const uint32_t xe = b * 256u + (m >> 1) * 64u + (m & 1u) * 16u;
        base[0] = xe, base[1] = xe + 32u, base[2] = 0, base[3] = 0;
        runs = 2, len = 16;
    } else {
        const uint32_t xe = b * 256u + (m >> 2) * 128u + 8u * (m & 3u);
        base[0] = xe, base[1] = xe + 32u, base[2] = xe + 64u, base[3] = xe + 96u;
        runs = 4, len = 8;
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        if (r < runs) {
            float t = 0.f;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                if (i < len) {
                    float v = x[base[r] + i];
                    if (gamma) v = (v * inv) * gamma[base[r] + i];
                    X.v[r * len + i] = v;
                    t += v;
                }
            }
            X.s[r] = t;
        } else {
            X.s[r] = 0.f;
        }
    }
}

template <int FMT, int G, bool DUAL, bool XREG, int NWC>
__global__ void __launch_bounds__((NWC + 1) * 32) matvec_stream_kernel(const MvParams p) {
    constexpr int NT = NWC * 32;
    constexpr int NV = DUAL ? 2 * G : G;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kMaxStages;
    int* cnt = reinterpret_cast<int*>(empty + kMaxStages);  // [kMaxStages]
    volatile int* abort_flag = cnt + kMaxStages;
    double* red_d = reinterpret_cast<double*>(smem + 2 * kMaxStages * 8 + 4 * kMaxStages + 16);  // [NWC]
    float* red = reinterpret_cast<float*>(red_d + NWC);  // [kMaxStages][NWC][NV]
    uint8_t* xsb = smem_align_up<16>(smem, (uint32_t)(reinterpret_cast<uint8_t*>(red + kMaxStages * NWC * NV) - smem));
    float* xs = reinterpret_cast<float*>(xsb);
    uint8_t* stages = smem_align_up<128>(smem, (uint32_t)(xsb - smem) + 4u * p.x_floats);

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    const uint32_t S = p.stages;
    const uint32_t mat_off = p.G * p.rb;  // offset of the second matrix inside a stage
    pdl_trigger();

    if (tid == NT) {
        for (uint32_t s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NWC);
            cnt[s] = 0;
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == NWC) {
        produce_groups<DUAL>(p, stages, full, empty, abort_flag, mat_off, lane);
        return;
    }

    // ---------------- consumer warps ----------------
    pdl_wait();  // x, gamma, bias and residual come from the preceding kernels
    // stage x once (optionally RMS-normalised as src/p8c_segmented_access_correctness.cpp:958-969)
    float inv = 1.0f;
    if (p.gamma) {
        double ss = 0.0;
        for (uint32_t i = tid; i < p.k; i += NT) {
            const double v = (double)p.x[i];
            ss += v * v;
        }
        ss = warp_sum_d(ss);
        if (lane == 0) red_d[warp] = ss;
        named_bar_sync(1, NT);
        double tot = 0.0;
#pragma unroll
        for (int w = 0; w < NWC; ++w) tot += red_d[w];
        inv = 1.0f / sqrtf((float)(tot / (double)p.k) + p.eps);
    }
    const uint32_t P = p.nb * 8u;  // 32-weight units per row
    UnitX X;
    if (XREG) {
        if (tid < P) load_unit_x_global<FMT>(p.x, p.gamma, inv, tid, X);
    } else {
        for (uint32_t i = tid; i < p.k; i += NT) {
            float v = p.x[i];
            if (p.gamma) v = (v * inv) * p.gamma[i];
            xs[xpad(i)] = v;
        }
        named_bar_sync(1, NT);
    }
    constexpr uint32_t kShift = 5u - (uint32_t)ilog2<NV>();

    uint32_t it = 0;
    for (uint32_t grp = blockIdx.x; grp < p.n_groups; grp += gridDim.x, ++it) {
        const uint32_t s = it % S;
        if (!mbar_wait(&full[s], (it / S) & 1u, p.err)) *abort_flag = 1;
        if (*abort_flag) break;
        const uint32_t rows_g = min(p.G, p.rows - grp * p.G);
        const uint8_t* st = stages + s * p.stage_smem;
        float acc[NV];
#pragma unroll
        for (int i = 0; i < NV; ++i) acc[i] = 0.f;
        if (XREG) {
            if (tid < P) apply_unit<FMT, G, DUAL>(st, mat_off, p.rb, rows_g, tid, X, acc);
        } else {
            for (uint32_t u = tid; u < P; u += NT) {
                load_unit_x<FMT>(xs, u, X);
                apply_unit<FMT, G, DUAL>(st, mat_off, p.rb, rows_g, u, X, acc);
            }
        }
        const float v = warp_fold<NV>(acc, lane);
        float* rs = red + s * NWC * NV;
        if ((lane & ((1u << kShift) - 1u)) == 0u) rs[warp * NV + (lane >> kShift)] = v;
        __syncwarp();
        int last = 0;
        if (lane == 0) {
            __threadfence_block();
            last = atomicAdd(&cnt[s], 1) == NWC - 1;
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            __threadfence_block();
            if (lane < rows_g) {
                const uint32_t row = grp * p.G + lane;
                float a = 0.f;
#pragma unroll
                for (int w = 0; w < NWC; ++w) a += rs[w * NV + lane];
                if (DUAL) {
                    float u = 0.f;
#pragma unroll
                    for (int w = 0; w < NWC; ++w) u += rs[w * NV + G + lane];
                    // src/p8c_segmented_access_correctness.cpp:1064-1073 (silu(g)*u)
                    p.y[row] = (a / (1.0f + expf(-a))) * u;
                } else {
                    if (p.bias) a += p.bias[row];
                    if (p.residual) a = p.residual[row] + a;
                    p.y[row] = a;
                }
            }
            if (lane == 0) cnt[s] = 0;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
}

struct DevInfo {
    int sms = 0;
    int max_smem = 0;
};

DevInfo dev_info() {
    static DevInfo cache[64];  // per device, queried once (under the mutex)
    static std::mutex mu;
    int dev = 0;
    cudaGetDevice(&dev);
    const int slot = device_slot();
    DevInfo d;
    if (slot >= 0) {
        std::lock_guard<std::mutex> lock(mu);
        d = cache[slot];
    }
    if (d.sms == 0) {
        cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
        cudaDeviceGetAttribute(&d.max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        if (slot >= 0) {
            std::lock_guard<std::mutex> lock(mu);
            cache[slot] = d;
        }
    }
    return d;
}

template <int FMT, int G, bool DUAL, bool XREG, int NWC>
cudaError_t set_attr() {
    return cudaFuncSetAttribute(matvec_stream_kernel<FMT, G, DUAL, XREG, NWC>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
}

template <int FMT, int G, bool DUAL>
cudaError_t set_attr_g() {
    cudaError_t e = set_attr<FMT, G, DUAL, true, 4>();
    if (e == cudaSuccess) e = set_attr<FMT, G, DUAL, true, 20>();
    if (e == cudaSuccess) e = set_attr<FMT, G, DUAL, false, 8>();
    return e;
}

// Opt every matvec instantiation into large dynamic shared memory on the
// current device (once).  Also forces the kernels to load, so launches can be
// captured into CUDA graphs afterwards.
cudaError_t prepare_all() {
    static std::atomic<bool> done[64] = {};  // concurrent first calls set the same (idempotent) attributes
    const int slot = device_slot();
    if (slot < 0) return cudaErrorInvalidDevice;
    if (done[slot].load(std::memory_order_acquire)) return cudaSuccess;
    cudaError_t e = set_attr_g<12, 4, false>();
    if (e == cudaSuccess) e = set_attr_g<12, 8, false>();
    if (e == cudaSuccess) e = set_attr_g<12, 16, false>();
    if (e == cudaSuccess) e = set_attr_g<12, 4, true>();
    if (e == cudaSuccess) e = set_attr_g<12, 8, true>();
    if (e == cudaSuccess) e = set_attr_g<14, 4, false>();
    if (e == cudaSuccess) e = set_attr_g<14, 8, false>();
    if (e == cudaSuccess) e = set_attr_g<14, 16, false>();
    if (e == cudaSuccess) done[slot].store(true, std::memory_order_release);
    return e;
}

template <int FMT, int G, bool DUAL, bool XREG, int NWC>
cudaError_t launch_t(const MvParams& p, uint32_t smem, uint32_t grid, cudaStream_t stream) {
    cudaError_t e = prepare_all();
    if (e != cudaSuccess) return e;
    return launch_kernel(matvec_stream_kernel<FMT, G, DUAL, XREG, NWC>, dim3(grid), dim3((NWC + 1) * 32), smem, stream,
                         p);
}

template <int FMT, int G, bool DUAL>
cudaError_t launch_g(const MatvecPlan& pl, const MvParams& p, cudaStream_t stream) {
    if (pl.xreg && pl.nwc == 4) return launch_t<FMT, G, DUAL, true, 4>(p, pl.smem, pl.grid, stream);
    if (pl.xreg && pl.nwc == 20) return launch_t<FMT, G, DUAL, true, 20>(p, pl.smem, pl.grid, stream);
    return launch_t<FMT, G, DUAL, false, 8>(p, pl.smem, pl.grid, stream);
}

uint32_t gcd_u(uint32_t a, uint32_t b) {
    while (b) {
        uint32_t t = a % b;
        a = b;
        b = t;
    }
    return a;
}

// Tuning override for experiments: ARCLLM_MATVEC_TUNE="<stage_kb>,<ctas_per_sm>"
void tune_override(uint32_t& target_stage, uint32_t& ctas) {
    static int parsed = 0;
    static unsigned kb = 0, c = 0;
    if (!parsed) {
        parsed = 1;
        if (const char* e = std::getenv("ARCLLM_MATVEC_TUNE")) std::sscanf(e, "%u,%u", &kb, &c);
    }
    if (kb) target_stage = kb * 1024u;
    if (c) ctas = c;
}

}  // namespace

int matvec_prepare() {
    const cudaError_t e = prepare_all();
    return e == cudaSuccess ? ARC_OK : set_cuda_error(e, "matvec prepare");
}

int matvec_plan(int fmt, bool dual, uint32_t rows, uint32_t k, MatvecPlan* out) {
    if (fmt != 12 && fmt != 14)
        return set_error(ARC_E_INVALID_ARGUMENT, "matvec: format must be Q4_K (12) or Q6_K (14)");
    if (dual && fmt != 12) return set_error(ARC_E_UNSUPPORTED_SHAPE, "matvec: the dual gate/up form is Q4_K only");
    if (rows == 0 || k == 0 || (k % 256u) != 0u)
        return set_error(ARC_E_INVALID_ARGUMENT, "matvec: rows must be >= 1 and k a non-zero multiple of 256");
    if (k > 32768u) return set_error(ARC_E_UNSUPPORTED_SHAPE, "matvec: k > 32768 is not supported");
    const uint32_t nb = k / 256u;
    const uint32_t rb = nb * (fmt == 12 ? 144u : 210u);
    const uint32_t gmin = fmt == 12 ? 1u : 8u / gcd_u(nb, 8u);
    const uint32_t mats = dual ? 2u : 1u;
    // x in registers when every consumer thread owns at most one 32-weight unit:
    // 4 consumer warps up to K = 4096, 20 up to K = 20480; beyond that 8 warps
    // loop over units with x staged in shared memory.
    const uint32_t units = nb * 8u;
    const bool xreg = units <= 640u;
    const uint32_t nwc = units <= 128u ? 4u : (xreg ? 20u : 8u);
    // measured on B200 (LM head / gate-up shapes): 4 CTAs per SM with ~24 KB
    // stages (two per CTA) keep enough consumer warps resident; the 20-warp
    // large-K form runs one CTA per SM with as many stages as fit.
    uint32_t target = 24u * 1024u;
    uint32_t ctas = nwc == 4u ? 4u : 1u;
    tune_override(target, ctas);
    // rows per stage: the largest of {4, 8, 16} (8 for the dual form) that is a
    // multiple of gmin and keeps a stage within `target` bytes (else the smallest)
    const uint32_t cand[3] = {4u, 8u, 16u};
    uint32_t G = 0;
    for (uint32_t c : cand) {
        if (c % gmin || (dual && c > 8u)) continue;
        if (G == 0 || c * rb * mats <= target) G = c;
    }
    if (G == 0) return set_error(ARC_E_UNSUPPORTED_SHAPE, "matvec: row group does not fit");
    const uint32_t GT = G;
    const uint32_t NV = GT * mats;
    const uint32_t stage_smem = ((G * rb * mats + kStagePad) + 127u) & ~127u;
    const uint32_t x_floats = xreg ? 0u : xpad_len(k);
    const uint32_t fixed = 2 * kMaxStages * 8 + 4 * kMaxStages + 16 + nwc * 8 + kMaxStages * nwc * NV * 4 + 16 +
                           x_floats * 4 + 128;
    const DevInfo di = dev_info();
    const uint32_t smem_cap = di.max_smem > 0 ? (uint32_t)di.max_smem : 227u * 1024u;
    int64_t S = 0;
    for (; ctas >= 1; --ctas) {
        const uint32_t budget = (228u * 1024u) / ctas - 1024u;
        S = ((int64_t)std::min(budget, smem_cap) - fixed) / stage_smem;
        if (S >= 2) break;
    }
    if (ctas < 1 || S < 2) return set_error(ARC_E_UNSUPPORTED_SHAPE, "matvec: not enough shared memory for two stages");
    if (S > kMaxStages) S = kMaxStages;
    out->fmt = fmt;
    out->dual = dual;
    out->xreg = xreg;
    out->nwc = nwc;
    out->rows = rows;
    out->k = k;
    out->nb = nb;
    out->rb = rb;
    out->G = G;
    out->gmax = GT;
    out->n_groups = (rows + G - 1u) / G;
    out->stages = (uint32_t)S;
    out->stage_smem = stage_smem;
    out->x_floats = x_floats;
    out->smem = fixed + (uint32_t)S * stage_smem;
    const uint32_t sms = di.sms > 0 ? (uint32_t)di.sms : 148u;
    out->grid = std::min(out->n_groups, sms * ctas);
    return ARC_OK;
}

int matvec_any(int fmt, bool dual, const void* w0, const void* w1, uint32_t rows, uint32_t k, const float* x,
               const float* gamma, float eps, const float* bias, const float* residual, float* y,
               cudaStream_t stream) {
    // Integer tensor-core kernels wherever their shape rules hold (16-byte
    // aligned x and gamma): whole rows for K <= 3584 (matvec_imma.cu), K
    // slices for K > 3584 (matvec_imma_splitk.cu; FFN down 3584 x 18944,
    // measured on B200: Q4_K 16.4 us against 27.5 us on CUDA cores, Q6_K
    // 20.7 us against 22.4 us); the CUDA-core streaming kernel otherwise.
    // ARCLLM_MATVEC_IMPL=cuda forces the CUDA-core kernel.
    const char* env = std::getenv("ARCLLM_MATVEC_IMPL");
    const int impl = (env && std::strcmp(env, "cuda") == 0) ? 0 : 1;
    const bool x_aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(gamma)) & 15u) == 0u;
    if (fmt == ARC_TYPE_EXEC148) {  // route B of the Q4 FFN-down capability
        if (dual || gamma || bias) return set_error(ARC_E_UNSUPPORTED_SHAPE, "matvec EXEC148: no gamma, bias or dual");
        // the K-slice integer-MMA kernel where its shape rules hold, else the CUDA-core kernel
        if (impl >= 1 && x_aligned && (reinterpret_cast<uintptr_t>(w0) & 15u) == 0u &&
            matvec_splitk_supported(fmt, false, rows, k))
            return matvec_splitk_launch(fmt, w0, rows, k, x, nullptr, 0.f, nullptr, residual, y, stream);
        return exec148_matvec(w0, rows, k, x, residual, y, stream);
    }
    if (impl >= 1 && x_aligned && matvec_imma_supported(fmt, dual, rows, k))
        return matvec_imma_launch(fmt, dual, w0, w1, rows, k, x, gamma, eps, bias, residual, y, stream);
    if (impl >= 1 && x_aligned && matvec_splitk_supported(fmt, dual, rows, k))
        return matvec_splitk_launch(fmt, w0, rows, k, x, gamma, eps, bias, residual, y, stream);
    MatvecPlan pl;
    int st = matvec_plan(fmt, dual, rows, k, &pl);
    if (st != ARC_OK) return st;
    return matvec_launch(pl, w0, w1, x, gamma, eps, bias, residual, y, stream);
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
    p.early = pdl_enabled() ? 1u : 0u;
    cudaError_t e;
    if (pl.fmt == 12) {
        if (pl.dual) {
            e = pl.gmax == 4 ? launch_g<12, 4, true>(pl, p, stream) : launch_g<12, 8, true>(pl, p, stream);
        } else {
            e = pl.gmax == 4   ? launch_g<12, 4, false>(pl, p, stream)
                : pl.gmax == 8 ? launch_g<12, 8, false>(pl, p, stream)
                               : launch_g<12, 16, false>(pl, p, stream);
        }
    } else {
        e = pl.gmax == 4   ? launch_g<14, 4, false>(pl, p, stream)
            : pl.gmax == 8 ? launch_g<14, 8, false>(pl, p, stream)
                           : launch_g<14, 16, false>(pl, p, stream);
    }
    if (e != cudaSuccess) return set_cuda_error(e, "matvec launch");
    return ARC_OK;
}

}  // namespace arc
