// M=1 dequant-matvec with the multiply-accumulate on the tensor cores
// (mma.sync m16n8k16, fp16 inputs, fp32 accumulate), for K <= 4096.
//
// Why: on B200 the CUDA-core kernel (matvec.cu) is limited by the integer
// work of turning packed codes into fp32 products (ALU pipe 60-70 % busy,
// ~14 weights/clk/SM, 26-43 % of HBM bandwidth; ncu).  Here a code becomes
// an exact fp16 integer with one LOP3 per two weights ((w & 0x000F000F) |
// 0x6400_6400 = 1024 + q, then one HADD2 removes the 1024), and the tensor
// core does the products.  Same streaming structure: a TMA producer warp
// fills a ring of whole-row stages; consumer warps own super-blocks.
//
// Exactness: A holds the integer codes exactly (Q4_K: q or 16q; Q6_K: q-32);
// x is split as x_hi = fp16(x), x_lo = fp16(x - x_hi) in two B columns, so
// each product is exact and the fp32 accumulators see (x_hi + x_lo) ~ x to
// 22 bits.  Sub-block scales are applied in fp32 after the MMAs.
//
// Layout trick: each MMA covers one K16 window of ONE scale sub-block, and the
// B operand puts that window's x_hi/x_lo into the column pair (2j, 2j+1) with
// j = sub-block mod 4 (zeros elsewhere).  Four consecutive sub-blocks then
// accumulate into one D fragment side by side, so after a super-block lane
// (g, t) holds, for rows g and g+8, the sums of the sub-blocks with index
// = t mod 4 -- every lane's accumulator is useful and the epilogue applies
// that lane's scales directly.
//
// Window element order (the same permutation in A and B, so no data moves
// between lanes): thread t of a quad contributes 4 consecutive codes of a
// 32-bit word per row; bytes 0,2 feed k = 2t, 2t+1 and bytes 1,3 feed
// k = 2t+8, 2t+9 -- the byte pairs a single LOP3 extracts.
#include <algorithm>

#include "arcllm_cuda_internal.h"
#include "common.cuh"
#include "matvec_common.cuh"

namespace arc {
namespace {

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// half2 arithmetic on raw bits: h - c (exact for the integer codes here)
__device__ __forceinline__ uint32_t hsub2_bits(uint32_t h, uint32_t c) {
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(h), "r"(c));
    return r;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    const uint32_t l = (uint32_t)__half_as_ushort(__float2half_rn(lo));
    const uint32_t h = (uint32_t)__half_as_ushort(__float2half_rn(hi));
    return l | (h << 16);
}

// x split for the B operand: column parity selects x_hi (even) or x_lo (odd)
__device__ __forceinline__ float x_part(float x, bool lo_part) {
    const float hi = __half2float(__float2half_rn(x));
    return lo_part ? (x - hi) : hi;
}

// 32-bit little-endian read at an even (possibly not 4-aligned) smem offset
__device__ __forceinline__ uint32_t lds32_even(const uint8_t* base, uint32_t off) {
    const uint32_t* p = reinterpret_cast<const uint32_t*>(base + (off & ~3u));
    return __funnelshift_r(p[0], p[1], (off & 3u) * 8u);
}

constexpr uint32_t kH1024 = 0x64006400u;  // half2(1024, 1024)
constexpr uint32_t kH1056 = 0x64206420u;  // half2(1056, 1056) = 1024 + 32

// ---- per-thread constants for one owned super-block --------------------
struct SbConst {
    uint32_t b[16][2];  // routed B fragments: window (sub-block s [, e]) -> (b0, b1)
    float xs[4];        // x sums of this lane's epilogue sub-blocks (Q4: t, 4+t)
};

template <int FMT>
__device__ __forceinline__ void make_sb_const(const float* x, const float* gamma, float inv, uint32_t b, uint32_t lane,
                                              SbConst& c) {
    const uint32_t g = lane >> 2, t = lane & 3u, j = g >> 1;
    const bool lo_part = (g & 1u) != 0;
    auto xn = [&](uint32_t e) {
        float v = x[e];
        if (gamma) v = (v * inv) * gamma[e];
        return v;
    };
    if (FMT == 12) {
        // window w = 2*s + e, s = sub-block 0..7, e = word 0/1 of the thread's pair
#pragma unroll
        for (int s = 0; s < 8; ++s) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                uint32_t b0 = 0, b1 = 0;
                if ((uint32_t)(s & 3) == j) {
                    const uint32_t base = b * 256u + 64u * (s >> 1) + 32u * (s & 1) + 8u * t + 4u * e;
                    b0 = pack_half2(x_part(xn(base + 0), lo_part), x_part(xn(base + 2), lo_part));
                    b1 = pack_half2(x_part(xn(base + 1), lo_part), x_part(xn(base + 3), lo_part));
                }
                c.b[2 * s + e][0] = b0;
                c.b[2 * s + e][1] = b1;
            }
        }
        // epilogue sub-blocks of this lane: t and 4+t (32 elements each)
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const uint32_t s = t + 4u * i;
            const uint32_t base = b * 256u + 64u * (s >> 1) + 32u * (s & 1u);
            float acc = 0.f;
            for (uint32_t k = 0; k < 32u; ++k) acc += xn(base + k);
            c.xs[i] = acc;
        }
        c.xs[2] = c.xs[3] = 0.f;
    } else {
        // window = sub-block s = 8h + 2q + lh; elements l = 16 lh + 4t + c of quarter q, half h
#pragma unroll
        for (int s = 0; s < 16; ++s) {
            uint32_t b0 = 0, b1 = 0;
            if ((uint32_t)(s & 3) == j) {
                const uint32_t h = s >> 3, q = (s >> 1) & 3, lh = s & 1;
                const uint32_t base = b * 256u + 128u * h + 32u * q + 16u * lh + 4u * t;
                b0 = pack_half2(x_part(xn(base + 0), lo_part), x_part(xn(base + 2), lo_part));
                b1 = pack_half2(x_part(xn(base + 1), lo_part), x_part(xn(base + 3), lo_part));
            }
            c.b[s][0] = b0;
            c.b[s][1] = b1;
        }
        c.xs[0] = c.xs[1] = c.xs[2] = c.xs[3] = 0.f;
    }
}

// ---- one 16-row M-tile x one super-block: returns the contribution to rows g, g+8
__device__ __forceinline__ void q4k_tile(const uint8_t* st, uint32_t r0off, uint32_t r1off, uint32_t t,
                                         const SbConst& c, float& y0, float& y1) {
    // four accumulators (sub-block group x word parity) so no MMA waits on the previous one's result
    float D0[4] = {0.f, 0.f, 0.f, 0.f}, D1[4] = {0.f, 0.f, 0.f, 0.f};
    float E0[4] = {0.f, 0.f, 0.f, 0.f}, E1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const uint2 w0 = *reinterpret_cast<const uint2*>(st + r0off + 16u + 32u * p + 8u * t);
        const uint2 w1 = *reinterpret_cast<const uint2*>(st + r1off + 16u + 32u * p + 8u * t);
        const uint32_t u0[2] = {w0.x, w0.y}, u1[2] = {w1.x, w1.y};
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const uint32_t s0 = u0[e] >> 8, s1 = u1[e] >> 8;
            // lo nibbles -> sub-block 2p (q), hi nibbles -> sub-block 2p+1 (16q)
            const uint32_t la0 = hsub2_bits((u0[e] & 0x000F000Fu) | kH1024, kH1024);
            const uint32_t la1 = hsub2_bits((u1[e] & 0x000F000Fu) | kH1024, kH1024);
            const uint32_t la2 = hsub2_bits((s0 & 0x000F000Fu) | kH1024, kH1024);
            const uint32_t la3 = hsub2_bits((s1 & 0x000F000Fu) | kH1024, kH1024);
            const uint32_t ha0 = hsub2_bits((u0[e] & 0x00F000F0u) | kH1024, kH1024);
            const uint32_t ha1 = hsub2_bits((u1[e] & 0x00F000F0u) | kH1024, kH1024);
            const uint32_t ha2 = hsub2_bits((s0 & 0x00F000F0u) | kH1024, kH1024);
            const uint32_t ha3 = hsub2_bits((s1 & 0x00F000F0u) | kH1024, kH1024);
            const int slo = 2 * p, shi = 2 * p + 1;
            float(&Dlo)[4] = (slo >> 2) ? (e ? E1 : D1) : (e ? E0 : D0);
            float(&Dhi)[4] = (shi >> 2) ? (e ? E1 : D1) : (e ? E0 : D0);
            mma16816(Dlo, la0, la1, la2, la3, c.b[2 * slo + e][0], c.b[2 * slo + e][1]);
            mma16816(Dhi, ha0, ha1, ha2, ha3, c.b[2 * shi + e][0], c.b[2 * shi + e][1]);
        }
    }
    // lane (g, t) holds sub-blocks t (D0) and 4+t (D1); odd t are hi-nibble sub-blocks (x16)
    const float f = (t & 1u) ? 0.0625f : 1.0f;
    const uint4 h0 = *reinterpret_cast<const uint4*>(st + r0off);
    const uint4 h1 = *reinterpret_cast<const uint4*>(st + r1off);
    const uint4 hh[2] = {h0, h1};
    float out[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const uint4 hd = hh[r];
        const float d = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xffffu)));
        const float dmin = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
        const uint32_t A = hd.y >> (8u * t), B = hd.z >> (8u * t), Cw = hd.w >> (8u * t);
        const float sc0 = (float)(A & 63u), mn0 = (float)(B & 63u);
        const float sc1 = (float)((Cw & 15u) | ((A >> 2) & 0x30u));
        const float mn1 = (float)(((Cw >> 4) & 15u) | ((B >> 2) & 0x30u));
        const float S0 = r ? ((D0[2] + D0[3]) + (E0[2] + E0[3])) : ((D0[0] + D0[1]) + (E0[0] + E0[1]));
        const float S1 = r ? ((D1[2] + D1[3]) + (E1[2] + E1[3])) : ((D1[0] + D1[1]) + (E1[0] + E1[1]));
        const float tt = fmaf(sc0, S0, sc1 * S1) * f;
        const float uu = fmaf(mn0, c.xs[0], mn1 * c.xs[1]);
        out[r] = fmaf(d, tt, -dmin * uu);
    }
    y0 += out[0];
    y1 += out[1];
}

__device__ __forceinline__ void q6k_tile(const uint8_t* st, uint32_t r0off, uint32_t r1off, uint32_t t,
                                         const SbConst& c, float& y0, float& y1) {
    float D[4][4], E[4][4];  // E takes the lh = 1 windows so consecutive MMAs are independent
#pragma unroll
    for (int i = 0; i < 4; ++i) D[i][0] = D[i][1] = D[i][2] = D[i][3] = E[i][0] = E[i][1] = E[i][2] = E[i][3] = 0.f;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int lh = 0; lh < 2; ++lh) {
            uint32_t v[2][4];
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const uint32_t ro = r ? r1off : r0off;
                const uint32_t qa = lds32_even(st, ro + 64u * h + 16u * lh + 4u * t);
                const uint32_t qb = lds32_even(st, ro + 64u * h + 32u + 16u * lh + 4u * t);
                const uint32_t qh = lds32_even(st, ro + 128u + 32u * h + 16u * lh + 4u * t);
                v[r][0] = (qa & 0x0F0F0F0Fu) | ((qh << 4) & 0x30303030u);
                v[r][1] = (qb & 0x0F0F0F0Fu) | ((qh << 2) & 0x30303030u);
                v[r][2] = ((qa >> 4) & 0x0F0F0F0Fu) | (qh & 0x30303030u);
                v[r][3] = ((qb >> 4) & 0x0F0F0F0Fu) | ((qh >> 2) & 0x30303030u);
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int s = 8 * h + 2 * q + lh;
                const uint32_t a0 = hsub2_bits((v[0][q] & 0x003F003Fu) | kH1024, kH1056);
                const uint32_t a1 = hsub2_bits((v[1][q] & 0x003F003Fu) | kH1024, kH1056);
                const uint32_t a2 = hsub2_bits(((v[0][q] >> 8) & 0x003F003Fu) | kH1024, kH1056);
                const uint32_t a3 = hsub2_bits(((v[1][q] >> 8) & 0x003F003Fu) | kH1024, kH1056);
                mma16816(lh ? E[s >> 2] : D[s >> 2], a0, a1, a2, a3, c.b[s][0], c.b[s][1]);
            }
        }
    }
    // lane (g, t) holds sub-blocks t, 4+t, 8+t, 12+t (D[0..3])
    float out[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const uint32_t ro = r ? r1off : r0off;
        const int8_t* scp = reinterpret_cast<const int8_t*>(st + ro + 192u + t);
        const float d = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(st + ro + 208u)));
        float tt = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float S = r ? ((D[i][2] + D[i][3]) + (E[i][2] + E[i][3])) : ((D[i][0] + D[i][1]) + (E[i][0] + E[i][1]));
            tt = fmaf((float)scp[4 * i], S, tt);
        }
        out[r] = d * tt;
    }
    y0 += out[0];
    y1 += out[1];
}

template <int FMT, int MT, bool DUAL>
__global__ void __launch_bounds__(15 * 32) matvec_mma_kernel(const MvParams p, uint32_t nwc) {
    constexpr int G = 16 * MT;
    constexpr int NV = DUAL ? 2 * G : G;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kMaxStages;
    int* cnt = reinterpret_cast<int*>(empty + kMaxStages);
    volatile int* abort_flag = cnt + kMaxStages;
    double* red_d = reinterpret_cast<double*>(smem + 2 * kMaxStages * 8 + 4 * kMaxStages + 16);  // [32]
    float* red = reinterpret_cast<float*>(red_d + 32);  // [stages][nwc][NV]
    uint8_t* stages = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(red + p.stages * nwc * NV) + 127) & ~uintptr_t(127));

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    const uint32_t NT = nwc * 32u;
    const uint32_t S = p.stages;
    const uint32_t mat_off = p.G * p.rb;

    if (tid == NT) {
        for (uint32_t s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], nwc);
            cnt[s] = 0;
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (warp == nwc) {
        produce_groups<DUAL>(p, stages, full, empty, abort_flag, mat_off, lane);
        return;
    }

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
        for (uint32_t w = 0; w < nwc; ++w) tot += red_d[w];
        inv = 1.0f / sqrtf((float)(tot / (double)p.k) + p.eps);
    }
    const uint32_t b = warp;  // one super-block per consumer warp
    const bool active = b < p.nb;
    SbConst C;
    if (active) make_sb_const<FMT>(p.x, p.gamma, inv, b, lane, C);
    const uint32_t g = lane >> 2, t = lane & 3u;
    const uint32_t bb = b * (FMT == 12 ? 144u : 210u);

    uint32_t it = 0;
    for (uint32_t grp = blockIdx.x; grp < p.n_groups; grp += gridDim.x, ++it) {
        const uint32_t s = it % S;
        if (!mbar_wait(&full[s], (it / S) & 1u, p.err)) *abort_flag = 1;
        if (*abort_flag) break;
        const uint32_t rows_g = min(p.G, p.rows - grp * p.G);
        const uint8_t* st = stages + s * p.stage_smem;
        float y[DUAL ? 2 : 1][MT][2];
#pragma unroll
        for (int mat = 0; mat < (DUAL ? 2 : 1); ++mat) {
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                y[mat][m][0] = y[mat][m][1] = 0.f;
                if (active) {
                    const uint32_t r0off = mat * mat_off + (16u * m + g) * p.rb + bb;
                    const uint32_t r1off = r0off + 8u * p.rb;
                    if (FMT == 12)
                        q4k_tile(st, r0off, r1off, t, C, y[mat][m][0], y[mat][m][1]);
                    else
                        q6k_tile(st, r0off, r1off, t, C, y[mat][m][0], y[mat][m][1]);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        // sum the quad's four lanes: lanes with t == 0 then hold rows g, g+8 of each tile
        float* rs = red + (s * nwc + warp) * NV;
#pragma unroll
        for (int mat = 0; mat < (DUAL ? 2 : 1); ++mat) {
#pragma unroll
            for (int m = 0; m < MT; ++m) {
#pragma unroll
                for (int r = 0; r < 2; ++r) {
                    float v = y[mat][m][r];
                    v += __shfl_xor_sync(0xffffffffu, v, 1);
                    v += __shfl_xor_sync(0xffffffffu, v, 2);
                    if (t == 0) rs[mat * G + 16 * m + 8 * r + g] = v;
                }
            }
        }
        __syncwarp();
        int last = 0;
        if (lane == 0) {
            __threadfence_block();
            last = atomicAdd(&cnt[s], 1) == (int)nwc - 1;
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            __threadfence_block();
            for (uint32_t r = lane; r < rows_g; r += 32u) {
                const uint32_t row = grp * p.G + r;
                float a = 0.f;
                for (uint32_t w = 0; w < nwc; ++w) a += red[(s * nwc + w) * NV + r];
                if (DUAL) {
                    float u = 0.f;
                    for (uint32_t w = 0; w < nwc; ++w) u += red[(s * nwc + w) * NV + G + r];
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
    }
}

template <int FMT, int MT, bool DUAL>
cudaError_t launch_mma_t(const MvParams& p, uint32_t nwc, uint32_t smem, uint32_t grid, cudaStream_t st) {
    matvec_mma_kernel<FMT, MT, DUAL><<<grid, (nwc + 1) * 32, smem, st>>>(p, nwc);
    return cudaGetLastError();
}

template <int FMT, int MT, bool DUAL>
cudaError_t set_attr_mma() {
    return cudaFuncSetAttribute(matvec_mma_kernel<FMT, MT, DUAL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                227 * 1024);
}

}  // namespace

int matvec_mma_prepare() {
    static bool done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (done[dev & 63]) return ARC_OK;
    cudaError_t e = set_attr_mma<12, 1, false>();
    if (e == cudaSuccess) e = set_attr_mma<12, 2, false>();
    if (e == cudaSuccess) e = set_attr_mma<12, 1, true>();
    if (e == cudaSuccess) e = set_attr_mma<14, 1, false>();
    if (e == cudaSuccess) e = set_attr_mma<14, 2, false>();
    if (e != cudaSuccess) return set_cuda_error(e, "matvec_mma prepare");
    done[dev & 63] = true;
    return ARC_OK;
}

// K <= 4096 (one super-block per consumer warp, at most 14 + 1 warps/CTA is
// the launch bound; K up to 16 super-blocks would need 17 warps, so cap at 14)
bool matvec_mma_supported(int fmt, bool dual, uint32_t rows, uint32_t k) {
    (void)rows;
    if (fmt != 12 && fmt != 14) return false;
    if (dual && fmt != 12) return false;
    return k % 256u == 0 && k / 256u >= 1 && k / 256u <= 14u;
}

int matvec_mma_launch(int fmt, bool dual, const void* w0, const void* w1, uint32_t rows, uint32_t k, const float* x,
                      const float* gamma, float eps, const float* bias, const float* residual, float* y,
                      cudaStream_t stream) {
    if (!matvec_mma_supported(fmt, dual, rows, k))
        return set_error(ARC_E_UNSUPPORTED_SHAPE, "matvec_mma: needs K/256 <= 14");
    if (!w0 || !x || !y || (dual && !w1)) return set_error(ARC_E_INVALID_ARGUMENT, "matvec: null pointer");
    if ((reinterpret_cast<uintptr_t>(w0) & 15u) || (w1 && (reinterpret_cast<uintptr_t>(w1) & 15u)))
        return set_error(ARC_E_ALIGNMENT, "matvec: weight pointers must be 16-byte aligned");
    int st = matvec_mma_prepare();
    if (st != ARC_OK) return st;
    const uint32_t nb = k / 256u;
    const uint32_t rb = nb * (fmt == 12 ? 144u : 210u);
    const uint32_t mats = dual ? 2u : 1u;
    // rows per stage: 32 (two M-tiles) when the stage stays <= 48 KB, else 16
    const uint32_t MT = (!dual && 32u * rb <= 48u * 1024u) ? 2u : 1u;
    const uint32_t G = 16u * MT;
    const uint32_t nwc = nb;
    const uint32_t NV = G * mats;
    const uint32_t stage_smem = ((G * rb * mats + kStagePad) + 127u) & ~127u;
    // two CTAs per SM with as many stages (<= 4) as fit
    const uint32_t budget = 113u * 1024u;
    const uint32_t fixed_base = 2 * kMaxStages * 8 + 4 * kMaxStages + 16 + 32 * 8 + 128;
    uint32_t S = 4;
    while (S > 2 && fixed_base + S * nwc * NV * 4u + S * stage_smem > budget) --S;
    const uint32_t smem = fixed_base + S * nwc * NV * 4u + S * stage_smem;
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
    p.rows = rows;
    p.k = k;
    p.nb = nb;
    p.rb = rb;
    p.G = G;
    p.n_groups = (rows + G - 1u) / G;
    p.stages = S;
    p.stage_smem = stage_smem;
    p.x_floats = 0;
    int sms = 148, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const uint32_t grid = std::min(p.n_groups, (uint32_t)sms * 2u);
    cudaError_t e;
    if (fmt == 12)
        e = dual ? launch_mma_t<12, 1, true>(p, nwc, smem, grid, stream)
                 : (MT == 2 ? launch_mma_t<12, 2, false>(p, nwc, smem, grid, stream)
                            : launch_mma_t<12, 1, false>(p, nwc, smem, grid, stream));
    else
        e = MT == 2 ? launch_mma_t<14, 2, false>(p, nwc, smem, grid, stream)
                    : launch_mma_t<14, 1, false>(p, nwc, smem, grid, stream);
    if (e != cudaSuccess) return set_cuda_error(e, "matvec_mma launch");
    return ARC_OK;
}

}  // namespace arc
