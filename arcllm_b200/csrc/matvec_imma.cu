// M=1 dequant-matvec on the tensor cores with integer MMA
// (mma.sync m16n8k32: u8 weight codes x s8 activation limbs -> s32), for
// K <= 14 super-blocks (3584).
//
// Why: the CUDA-core kernel (matvec.cu) spends ~9 lane-instructions per
// weight turning packed codes into fp32 products and saturates the ALU pipe
// at ~14 weights/clk/SM.  Here the codes go to the tensor core as they are:
// a Q4_K byte pair becomes MMA operands with one LOP3 per four weights
// (w & 0x0F0F0F0F and w & 0xF0F0F0F0), a Q6_K code with ~3 logic ops per four
// weights, and one MMA multiplies 512 codes.
//
// Activations: each 32-element block of x (after the fused RMSNorm) is held
// as a 22-bit fixed-point integer with a power-of-two scale 2^e chosen from
// the block's max |x| (x_int = rint(x * 2^-e), |x_int| < 2^22, e >= -140), split into
// three signed 8-bit limbs x_int = 65536*l0 + 256*l1 + l2.  The MMAs give the
// exact integer sums S_L = sum(q * l_L) per scale group; the epilogue forms
// (256*(256*S_0 + S_1) + S_2) in fp32 and applies d, the group scale and 2^e.
// The only rounding beyond the fp32 epilogue is x's quantisation, at most
// 2^-22 of the block's max |x| -- the precision of fp32 itself.  Non-finite x
// makes the block's scale NaN, so the output row is NaN as in the reference.
//
// Column routing: every MMA covers one k32 window of ONE weight row-tile; the
// B operand puts a scale group's limbs into its own column pair (limbs 0,1 in
// one MMA, limb 2 in a second MMA) and zeros elsewhere, so the four column
// pairs of a D fragment collect four different groups.  Lane (g, t) then
// holds, for rows g and g+8, the sums of group(s) number t of every D, and
// applies that group's scales itself -- no lane's accumulator is wasted.
//
// Work split: a TMA producer warp streams groups of 16*MT whole rows into a
// shared-memory ring; consumer warp w owns super-block w (Q6_K: half of
// block w and half of block w^1, so every warp sees the same shared-memory
// alignment mix) for the whole kernel, so its B fragments (the routed x
// limbs) and scale constants stay in registers.  Consumers leave per-row
// partials in shared memory; the producer warp adds them in a fixed warp
// order (deterministic) after refilling the stage.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>

#include "arcllm_cuda_internal.h"
#include "common.cuh"
#include "matvec_common.cuh"

namespace arc {
namespace {

constexpr uint32_t kXScratch = 1024;  // per consumer warp: 3 limb planes x 256 B + block constants
constexpr uint32_t kRedD = 2 * kMaxStages * 8 + 4 * kMaxStages + 16;  // 176: after barriers, counters, flag

__host__ __device__ constexpr uint32_t imma_xscr_off(uint32_t S, uint32_t nwc, uint32_t NV) {
    return (kRedD + 32 * 8 + 2 * S * nwc * NV * 4 + 15u) & ~15u;  // row partials double-buffered
}
__host__ __device__ constexpr uint32_t imma_stage_off(uint32_t S, uint32_t nwc, uint32_t NV) {
    return imma_xscr_off(S, nwc, NV) + nwc * kXScratch;
}

// D += A * B, A 16x32 u8 (row), B 32x8 s8 (col), D s32
__device__ __forceinline__ void imma(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                     uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// (256 * (256*c0 + c1 - h) + (c2 - l)) in fp32; the integer parts are exact
__device__ __forceinline__ float combine(int c0, int c1, int c2, int h, int l) {
    return fmaf((float)(c0 * 256 + c1 - h), 256.0f, (float)(c2 - l));
}

// 32-bit read at a smem offset that is 4-aligned (EVEN) or 2 mod 4 (ODD)
template <bool ODD>
__device__ __forceinline__ uint32_t ld32(const uint8_t* base, uint32_t off) {
    if (!ODD) return *reinterpret_cast<const uint32_t*>(base + off);
    const uint32_t* q = reinterpret_cast<const uint32_t*>(base + (off & ~3u));
    return __funnelshift_r(q[0], q[1], 16);
}

// Per-lane state that depends only on x and the warp's super-block.
struct XFrag {
    uint32_t b1[8][2];  // limbs 0/1 routed to column pairs (k32 window m -> fragment m)
    uint32_t b2[8][2];  // limb 2 routed to the even column of the pair
    float sx[4];        // Q4: [0..1] scale of sub-blocks t, 4+t (x 1/16 for high nibbles); Q6: [0..3] per group
    float xs[2];        // Q4: sum of x over sub-blocks t, 4+t (dmin term)
    int xh[4], xl[4];   // Q6: 32 * (256*sum l0 + sum l1), 32 * sum l2 over group 4i+t
};

// pack the low bytes of four ints
__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
    return __byte_perm(__byte_perm((uint32_t)a, (uint32_t)b, 0x0040), __byte_perm((uint32_t)c, (uint32_t)d, 0x0040),
                       0x5410);
}

// Quantise the warp's 256 x values (windows 0..3 from block bA, 4..7 from
// block bB) into limb planes (smem), then gather this lane's routed B
// fragments and epilogue constants.  Lane L quantises elements 8(L&3)..+7 of
// window L>>2, so block reductions take two quad shuffles.
template <int FMT>
__device__ __forceinline__ void build_xfrag(const float* x, const float* gamma, float eps, uint32_t k, double* red_d,
                                            uint32_t nwc, uint32_t warp, uint32_t bA, uint32_t bB, uint32_t lane,
                                            uint8_t* xs, XFrag& f) {
    uint8_t* plane = xs;                                  // [3][256] int8 limbs
    float* kc = reinterpret_cast<float*>(xs + 768);       // [8][6]: sx, sum, xh(lh0), xl(lh0), xh(lh1), xl(lh1)
    const uint32_t jw = lane >> 2, qd = lane & 3u;        // window, quarter of the window
    const uint32_t e0 = 256u * (jw < 4 ? bA : bB) + 32u * jw + 8u * qd;
    float v[8];
    {
        const float4 a0 = *reinterpret_cast<const float4*>(x + e0);
        const float4 a1 = *reinterpret_cast<const float4*>(x + e0 + 4);
        v[0] = a0.x, v[1] = a0.y, v[2] = a0.z, v[3] = a0.w, v[4] = a1.x, v[5] = a1.y, v[6] = a1.z, v[7] = a1.w;
    }
    if (gamma) {
        const float4 g0 = *reinterpret_cast<const float4*>(gamma + e0);
        const float4 g1 = *reinterpret_cast<const float4*>(gamma + e0 + 4);
        const float gv[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
        // fused RMSNorm: 1/sqrt(mean(x^2) + eps), sum of squares in double.
        // The warps' 256-element slices cover x exactly once.
        double ss = 0.0;
#pragma unroll
        for (int i = 0; i < 8; ++i) ss += (double)v[i] * (double)v[i];
        ss = warp_sum_d(ss);
        if (lane == 0) red_d[warp] = ss;
        named_bar_sync(1, nwc * 32u);
        double tot = 0.0;
        for (uint32_t w = 0; w < nwc; ++w) tot += red_d[w];
        const float inv = 1.0f / sqrtf((float)(tot / (double)k) + eps);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = (v[i] * inv) * gv[i];
    }
    float a = 0.f;
    bool fin = true;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float m = fabsf(v[i]);
        fin = fin && (m <= 3.402823466e38f);  // false for inf and NaN
        a = fmaxf(a, m);
    }
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 2));
    const bool all_finite = ((__ballot_sync(0xffffffffu, !fin) >> (lane & ~3u)) & 15u) == 0u;
    // block exponent: a = m * 2^E, m in [0.5, 1) (E = -125 for zero or subnormal a);
    // x_int = rint(v * 2^-sh) with |x_int| < 2^22; powers of two keep the
    // scaling exact.  Blocks below 2^-118 take the scale in two steps and
    // keep a subnormal 2^sh (exact down to 2^-149).
    const uint32_t be = (__float_as_uint(a) >> 23) & 255u;
    const int E = all_finite ? (be ? (int)be - 126 : -125) : 0;
    const int sh = max(E - 22, -140);
    int ds = -sh;
    float pre = 1.0f;
    if (ds > 100) {
        pre = 18446744073709551616.0f;  // 2^64
        ds -= 64;
    }
    const float down = __int_as_float((127 + ds) << 23);
    int l0[8], l1[8], l2[8];
    int xh = 0, xl = 0;
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int xi = all_finite ? __float2int_rn((v[i] * pre) * down) : 0;
        l2[i] = ((xi + 128) & 255) - 128;
        const int r1 = (xi - l2[i]) >> 8;
        l1[i] = ((r1 + 128) & 255) - 128;
        l0[i] = (r1 - l1[i]) >> 8;
        xh += 256 * l0[i] + l1[i];
        xl += l2[i];
        sum += v[i];
    }
    const uint32_t o = 32u * jw + 8u * qd;
    *reinterpret_cast<uint2*>(plane + o) = make_uint2(pack4(l0[0], l0[1], l0[2], l0[3]), pack4(l0[4], l0[5], l0[6], l0[7]));
    *reinterpret_cast<uint2*>(plane + 256 + o) =
        make_uint2(pack4(l1[0], l1[1], l1[2], l1[3]), pack4(l1[4], l1[5], l1[6], l1[7]));
    *reinterpret_cast<uint2*>(plane + 512 + o) =
        make_uint2(pack4(l2[0], l2[1], l2[2], l2[3]), pack4(l2[4], l2[5], l2[6], l2[7]));
    if (FMT == 12) {
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    } else {  // 16-element scale groups: lanes (q, q^1) of a window share one
        xh += __shfl_xor_sync(0xffffffffu, xh, 1);
        xl += __shfl_xor_sync(0xffffffffu, xl, 1);
    }
    if (qd == 0) {
        const float sxv = sh >= -126 ? __int_as_float((127 + sh) << 23) : __int_as_float(1 << (149 + sh));
        kc[6 * jw + 0] = all_finite ? sxv : __int_as_float(0x7fc00000);
        kc[6 * jw + 1] = sum;
    }
    if (qd == 0 || qd == 2) {
        kc[6 * jw + 2 + qd] = __int_as_float(xh);
        kc[6 * jw + 3 + qd] = __int_as_float(xl);
    }
    __syncwarp();
    const uint32_t g = lane >> 2, t = lane & 3u, c = g >> 1, L = g & 1u;
    const uint8_t* pl = xs + 256u * L;
    const uint8_t* p2 = xs + 512u;
    if (FMT == 12) {
        // window m = sub-block s; slots 4t..4t+3 <- elements 8t..8t+3, slots 16+4t.. <- 8t+4..8t+7.
        // This lane's nonzero windows are s = c and c + 4.
        uint2 w1[2], w2[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t off = 32u * (c + 4u * h) + 8u * t;
            w1[h] = *reinterpret_cast<const uint2*>(pl + off);
            w2[h] = L == 0 ? *reinterpret_cast<const uint2*>(p2 + off) : make_uint2(0u, 0u);
        }
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            const bool on = (uint32_t)(s & 3) == c;
            f.b1[s][0] = on ? w1[s >> 2].x : 0u;
            f.b1[s][1] = on ? w1[s >> 2].y : 0u;
            f.b2[s][0] = on ? w2[s >> 2].x : 0u;
            f.b2[s][1] = on ? w2[s >> 2].y : 0u;
        }
        const float hi = (t & 1u) ? 0.0625f : 1.0f;  // odd sub-blocks use the 16*q high-nibble codes
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const uint32_t sb = 4u * i + t;
            f.sx[i] = kc[6 * sb] * hi;
            f.xs[i] = kc[6 * sb + 1];
        }
        f.sx[2] = f.sx[3] = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) f.xh[i] = f.xl[i] = 0;
    } else {
        // window m = 4h + q (quarter q of half h); slot k <- element l = k; groups lh = k >> 4
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            const int q = m & 3;
            const bool on0 = c == 2u * (q & 1), on1 = c == 2u * (q & 1) + 1u;
            const uint32_t off = 32u * m + 4u * t;
            f.b1[m][0] = on0 ? *reinterpret_cast<const uint32_t*>(pl + off) : 0u;
            f.b1[m][1] = on1 ? *reinterpret_cast<const uint32_t*>(pl + off + 16) : 0u;
            f.b2[m][0] = (on0 && L == 0) ? *reinterpret_cast<const uint32_t*>(p2 + off) : 0u;
            f.b2[m][1] = (on1 && L == 0) ? *reinterpret_cast<const uint32_t*>(p2 + off + 16) : 0u;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t j = 4u * (i >> 1) + 2u * (i & 1) + (t >> 1), lh = t & 1u;
            f.sx[i] = kc[6 * j];
            f.xh[i] = 32 * __float_as_int(kc[6 * j + 2 + 2 * lh]);
            f.xl[i] = 32 * __float_as_int(kc[6 * j + 3 + 2 * lh]);
        }
        f.xs[0] = f.xs[1] = 0.f;
    }
}

// One 16-row tile x one Q4_K super-block: adds the rows' partial dot products
// (this lane's sub-blocks t and 4+t) to y0 (row g) and y1 (row g+8).
__device__ __forceinline__ void q4_tile(const uint8_t* st, uint32_t r0, uint32_t r1, uint32_t t, const XFrag& f,
                                        float& y0, float& y1) {
    int D1[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}}, D2[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const uint2 w0 = *reinterpret_cast<const uint2*>(st + r0 + 16u + 32u * p + 8u * t);
        const uint2 w1 = *reinterpret_cast<const uint2*>(st + r1 + 16u + 32u * p + 8u * t);
        const int i = p >> 1, slo = 2 * p, shi = 2 * p + 1;
        const uint32_t l0 = w0.x & 0x0F0F0F0Fu, l1 = w1.x & 0x0F0F0F0Fu, l2 = w0.y & 0x0F0F0F0Fu,
                       l3 = w1.y & 0x0F0F0F0Fu;
        const uint32_t h0 = w0.x & 0xF0F0F0F0u, h1 = w1.x & 0xF0F0F0F0u, h2 = w0.y & 0xF0F0F0F0u,
                       h3 = w1.y & 0xF0F0F0F0u;
        imma(D1[i], l0, l1, l2, l3, f.b1[slo][0], f.b1[slo][1]);
        imma(D2[i], l0, l1, l2, l3, f.b2[slo][0], f.b2[slo][1]);
        imma(D1[i], h0, h1, h2, h3, f.b1[shi][0], f.b1[shi][1]);
        imma(D2[i], h0, h1, h2, h3, f.b2[shi][0], f.b2[shi][1]);
    }
    const uint4 hh[2] = {*reinterpret_cast<const uint4*>(st + r0), *reinterpret_cast<const uint4*>(st + r1)};
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
        const float F0 = combine(D1[0][2 * r], D1[0][2 * r + 1], D2[0][2 * r], 0, 0);
        const float F1 = combine(D1[1][2 * r], D1[1][2 * r + 1], D2[1][2 * r], 0, 0);
        const float tt = fmaf(sc0 * f.sx[0], F0, (sc1 * f.sx[1]) * F1);
        const float uu = fmaf(mn0, f.xs[0], mn1 * f.xs[1]);
        out[r] = fmaf(d, tt, -dmin * uu);
    }
    y0 += out[0];
    y1 += out[1];
}

// One 16-row tile x one Q6_K "super-block" made of two half-blocks: half 0
// (ql[0..63], qh[0..31], scales 0..7) of block bA and half 1 of block bB.
// bA and bB have opposite parity, so every warp does one 4-byte-aligned half
// and one half at 2 mod 4 in shared memory (ODD0: half 0 is the odd one).
template <bool ODD0>
__device__ __forceinline__ void q6_tile(const uint8_t* st, uint32_t row0, uint32_t row1, uint32_t offA, uint32_t offB,
                                        uint32_t t, const XFrag& f, float& y0, float& y1) {
    int D1[4][4], D2[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) D1[i][j] = D2[i][j] = 0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        constexpr bool kOddFirst = ODD0;
        const bool odd = (h == 0) ? kOddFirst : !kOddFirst;
        const uint32_t boff = h ? offB : offA;
        uint32_t v[2][2][4];  // [lh][row][quarter]: 4 codes (l = 16lh + 4t .. +3) as u8 in [0, 63]
#pragma unroll
        for (int lh = 0; lh < 2; ++lh) {
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const uint32_t ro = (r ? row1 : row0) + boff + 16u * lh + 4u * t;
                uint32_t qa, qb, qh;
                if (odd) {
                    qa = ld32<true>(st, ro + 64u * h);
                    qb = ld32<true>(st, ro + 64u * h + 32u);
                    qh = ld32<true>(st, ro + 128u + 32u * h);
                } else {
                    qa = ld32<false>(st, ro + 64u * h);
                    qb = ld32<false>(st, ro + 64u * h + 32u);
                    qh = ld32<false>(st, ro + 128u + 32u * h);
                }
                v[lh][r][0] = (qa & 0x0F0F0F0Fu) | ((qh << 4) & 0x30303030u);
                v[lh][r][1] = (qb & 0x0F0F0F0Fu) | ((qh << 2) & 0x30303030u);
                v[lh][r][2] = ((qa >> 4) & 0x0F0F0F0Fu) | (qh & 0x30303030u);
                v[lh][r][3] = ((qb >> 4) & 0x0F0F0F0Fu) | ((qh >> 2) & 0x30303030u);
            }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int m = 4 * h + q, i = 2 * h + (q >> 1);
            imma(D1[i], v[0][0][q], v[0][1][q], v[1][0][q], v[1][1][q], f.b1[m][0], f.b1[m][1]);
            imma(D2[i], v[0][0][q], v[0][1][q], v[1][0][q], v[1][1][q], f.b2[m][0], f.b2[m][1]);
        }
    }
    float out[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const uint32_t ro = r ? row1 : row0;
        float part[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            // group 4i + t of half h lives in block h ? bB : bA (scales 8h..8h+7)
            const int8_t* sc = reinterpret_cast<const int8_t*>(st + ro + (h ? offB : offA) + 192u + t);
            float acc = 0.f;
#pragma unroll
            for (int ii = 0; ii < 2; ++ii) {
                const int i = 2 * h + ii;
                const float F = combine(D1[i][2 * r], D1[i][2 * r + 1], D2[i][2 * r], f.xh[i], f.xl[i]);
                acc = fmaf((float)sc[4 * i] * f.sx[i], F, acc);
            }
            part[h] = acc;
        }
        const float dA = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(st + ro + offA + 208u)));
        const float dB = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(st + ro + offB + 208u)));
        out[r] = fmaf(dA, part[0], dB * part[1]);
    }
    y0 += out[0];
    y1 += out[1];
}

// Stage-local rows of M-tile m: (row of lanes g, row of lanes g+8).  For Q6_K
// with two tiles the rows are interleaved (4g+m, 4g+2+m) so that the eight
// row groups of a 32-bit shared-memory read fall into different banks
// (row stride 2940 B = -1 word mod 32 banks).
template <int FMT, int MT>
__device__ __forceinline__ uint2 tile_rows(int m, uint32_t g) {
    if (FMT == 14 && MT == 2) return make_uint2(4u * g + m, 4u * g + 2u + m);
    return make_uint2(16u * m + g, 16u * m + g + 8u);
}

// Final row sums of one finished stage round `itr`: the consumer warps' partials
// (red[parity][slot][warp][row]) added in warp order, plus bias / residual or
// the SiLU(gate)*up product, written to y.  Run by the producer warp.
template <int G, bool DUAL>
__device__ __forceinline__ void finish_rows(const MvParams& p, const float* red, uint32_t nwc, uint32_t itr,
                                            uint32_t lane) {
    constexpr int NV = DUAL ? 2 * G : G;
    const uint32_t S = p.stages, s = itr % S, par = (itr / S) & 1u;
    const uint32_t grp = blockIdx.x + itr * gridDim.x;
    const uint32_t rows_g = min(p.G, p.rows - grp * p.G);
    const float* rs = red + (par * S + s) * nwc * NV;
    for (uint32_t r = lane; r < rows_g; r += 32u) {
        const uint32_t row = grp * p.G + r;
        float a = 0.f;
        for (uint32_t w = 0; w < nwc; ++w) a += rs[w * NV + r];
        if (DUAL) {
            float u = 0.f;
            for (uint32_t w = 0; w < nwc; ++w) u += rs[w * NV + G + r];
            // src/p8c_segmented_access_correctness.cpp:1064-1073 (silu(g)*u)
            p.y[row] = (a / (1.0f + expf(-a))) * u;
        } else {
            if (p.bias) a += p.bias[row];
            if (p.residual) a = p.residual[row] + a;
            p.y[row] = a;
        }
    }
}

// The producer warp: stream row groups into the stage ring (1-D TMA bulk
// copies, as produce_groups does), and once the consumers release a stage,
// refill it first and then finish that stage's rows from their partials.
// Partials are double-buffered by round parity, so a consumer writing round
// r+1 never touches the buffer of round r being summed here.  All waits are
// bounded; on a timeout it sets *abort_flag, stops, and waits (bounded) for
// the copies it already issued.
template <int G, bool DUAL>
__device__ __forceinline__ void produce_and_finish(const MvParams& p, uint8_t* stages, uint64_t* full,
                                                   uint64_t* empty, volatile int* abort_flag, uint32_t mat_off,
                                                   const float* red, uint32_t nwc, uint32_t lane) {
    const uint32_t S = p.stages;
    const uint64_t pol = l2_evict_first_policy();
    uint32_t it = 0;
    bool ok = true;
    auto released = [&](uint32_t j) {  // wait until the consumers released round j of its slot
        bool w = true;
        if (lane == 0) w = mbar_wait(&empty[j % S], (j / S) & 1u, p.err);
        w = __shfl_sync(0xffffffffu, w, 0);
        if (!w || *abort_flag) {
            if (lane == 0) *abort_flag = 1;
            return false;
        }
        return true;
    };
    for (uint32_t grp = blockIdx.x; grp < p.n_groups; grp += gridDim.x, ++it) {
        const uint32_t s = it % S;
        if (it >= S && !released(it - S)) {
            ok = false;
            break;
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
        if (it >= S) finish_rows<G, DUAL>(p, red, nwc, it - S, lane);
    }
    if (ok) {
        for (uint32_t j = it > S ? it - S : 0; j < it; ++j) {
            if (!released(j)) {
                ok = false;
                break;
            }
            finish_rows<G, DUAL>(p, red, nwc, j, lane);
        }
    }
    // on abort: no bulk copy may still be landing in this CTA's smem at exit
    if (!ok && lane == 0) {
        const uint32_t first = it > S ? it - S : 0;
        for (uint32_t j = first; j < it; ++j) mbar_wait(&full[j % S], (j / S) & 1u, p.err);
    }
}

template <int FMT, int MT, bool DUAL>
__global__ void __launch_bounds__(15 * 32, 1) matvec_imma_kernel(const MvParams p, uint32_t nwc) {
    constexpr int G = 16 * MT;
    constexpr int NV = DUAL ? 2 * G : G;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kMaxStages;
    int* cnt = reinterpret_cast<int*>(empty + kMaxStages);
    volatile int* abort_flag = cnt + kMaxStages;
    double* red_d = reinterpret_cast<double*>(smem + kRedD);  // [32]
    float* red = reinterpret_cast<float*>(red_d + 32);        // [2][stages][nwc][NV]
    uint8_t* xscr = smem + imma_xscr_off(p.stages, nwc, NV);
    uint8_t* stages = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem + imma_stage_off(p.stages, nwc, NV)) + 127) & ~uintptr_t(127));

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
        produce_and_finish<G, DUAL>(p, stages, full, empty, abort_flag, mat_off, red, nwc, lane);
        return;
    }

    // Q4_K: warp w owns super-block w.  Q6_K: half 0 of block w and half 1 of
    // block w^1 (K has an even number of blocks), see q6_tile.
    const uint32_t bA = warp, bB = (FMT == 14) ? (warp ^ 1u) : warp;
    XFrag f;
    build_xfrag<FMT>(p.x, p.gamma, p.eps, p.k, red_d, nwc, warp, bA, bB, lane, xscr + warp * kXScratch, f);
    const uint32_t g = lane >> 2, t = lane & 3u;
    const uint32_t bsz = FMT == 12 ? 144u : 210u;
    const uint32_t offA = bA * bsz, offB = bB * bsz;
    const bool oddA = FMT == 14 && (offA & 3u) != 0u;

    uint32_t it = 0;
    for (uint32_t grp = blockIdx.x; grp < p.n_groups; grp += gridDim.x, ++it) {
        const uint32_t s = it % S;
        if (!mbar_wait(&full[s], (it / S) & 1u, p.err)) *abort_flag = 1;
        if (*abort_flag) break;
        const uint8_t* st = stages + s * p.stage_smem;
        float y[DUAL ? 2 : 1][MT][2];
#pragma unroll
        for (int mat = 0; mat < (DUAL ? 2 : 1); ++mat) {
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                y[mat][m][0] = y[mat][m][1] = 0.f;
                const uint2 rr = tile_rows<FMT, MT>(m, g);
                const uint32_t row0 = mat * mat_off + rr.x * p.rb;
                const uint32_t row1 = mat * mat_off + rr.y * p.rb;
                if (FMT == 12)
                    q4_tile(st, row0 + offA, row1 + offA, t, f, y[mat][m][0], y[mat][m][1]);
                else if (oddA)
                    q6_tile<true>(st, row0, row1, offA, offB, t, f, y[mat][m][0], y[mat][m][1]);
                else
                    q6_tile<false>(st, row0, row1, offA, offB, t, f, y[mat][m][0], y[mat][m][1]);
            }
        }
        // sum the quad's four lanes; lanes t == 0 then hold the warp's partial of rows g, g+8
        float* rs = red + (((it / S) & 1u) * S + s) * nwc * NV + warp * NV;
#pragma unroll
        for (int mat = 0; mat < (DUAL ? 2 : 1); ++mat) {
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                const uint2 rr = tile_rows<FMT, MT>(m, g);
#pragma unroll
                for (int r = 0; r < 2; ++r) {
                    float v = y[mat][m][r];
                    v += __shfl_xor_sync(0xffffffffu, v, 1);
                    v += __shfl_xor_sync(0xffffffffu, v, 2);
                    if (t == 0) rs[mat * G + (r ? rr.y : rr.x)] = v;
                }
            }
        }
        __syncwarp();
        if (lane == 0) {
            __threadfence_block();
            mbar_arrive(&empty[s]);  // releases the stage and publishes this warp's partials
        }
    }
}

template <int FMT, int MT, bool DUAL>
cudaError_t launch_imma_t(const MvParams& p, uint32_t nwc, uint32_t smem, uint32_t grid, cudaStream_t st) {
    matvec_imma_kernel<FMT, MT, DUAL><<<grid, (nwc + 1) * 32, smem, st>>>(p, nwc);
    return cudaGetLastError();
}

template <int FMT, int MT, bool DUAL>
cudaError_t set_attr_imma() {
    return cudaFuncSetAttribute(matvec_imma_kernel<FMT, MT, DUAL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                227 * 1024);
}

struct ImmaConfig {
    uint32_t MT, G, S, stage_smem, smem;
};

// Tuning override for experiments: ARCLLM_IMMA_TUNE="<MT>,<max stages>"
void imma_tune(uint32_t& mt, uint32_t& smax) {
    static int parsed = 0;
    static unsigned m = 0, s = 0;
    if (!parsed) {
        parsed = 1;
        if (const char* e = std::getenv("ARCLLM_IMMA_TUNE")) std::sscanf(e, "%u,%u", &m, &s);
    }
    if (m == 1 || m == 2) mt = m;
    if (s >= 2 && s <= (unsigned)kMaxStages) smax = s;
}

ImmaConfig imma_config(int fmt, bool dual, uint32_t k) {
    const uint32_t nb = k / 256u, rb = nb * (fmt == 12 ? 144u : 210u), mats = dual ? 2u : 1u;
    ImmaConfig c{};
    c.MT = (32u * rb * mats <= 100u * 1024u) ? 2u : 1u;
    uint32_t smax = kMaxStages;
    imma_tune(c.MT, smax);
    c.G = 16u * c.MT;
    c.stage_smem = ((c.G * rb * mats + kStagePad) + 127u) & ~127u;
    const uint32_t NV = c.G * mats;
    const uint32_t budget = 227u * 1024u;
    uint32_t S = smax;
    while (S > 2 && imma_stage_off(S, nb, NV) + 128u + S * c.stage_smem > budget) --S;
    c.S = S;
    c.smem = imma_stage_off(S, nb, NV) + 128u + S * c.stage_smem;
    return c;
}

}  // namespace

int matvec_imma_prepare() {
    static bool done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (done[dev & 63]) return ARC_OK;
    cudaError_t e = set_attr_imma<12, 1, false>();
    if (e == cudaSuccess) e = set_attr_imma<12, 2, false>();
    if (e == cudaSuccess) e = set_attr_imma<12, 1, true>();
    if (e == cudaSuccess) e = set_attr_imma<12, 2, true>();
    if (e == cudaSuccess) e = set_attr_imma<14, 1, false>();
    if (e == cudaSuccess) e = set_attr_imma<14, 2, false>();
    if (e != cudaSuccess) return set_cuda_error(e, "matvec_imma prepare");
    done[dev & 63] = true;
    return ARC_OK;
}

// One consumer warp per super-block (K <= 3584); Q6_K rows must keep their
// blocks at a fixed 4-byte phase in shared memory (even number of blocks).
bool matvec_imma_supported(int fmt, bool dual, uint32_t rows, uint32_t k) {
    if (fmt != 12 && fmt != 14) return false;
    if (dual && fmt != 12) return false;
    if (rows == 0 || k % 256u) return false;
    const uint32_t nb = k / 256u;
    if (nb < 1 || nb > 14) return false;
    if (fmt == 14 && (nb & 1u)) return false;
    return imma_config(fmt, dual, k).smem <= 227u * 1024u;
}

int matvec_imma_launch(int fmt, bool dual, const void* w0, const void* w1, uint32_t rows, uint32_t k, const float* x,
                       const float* gamma, float eps, const float* bias, const float* residual, float* y,
                       cudaStream_t stream) {
    if (!matvec_imma_supported(fmt, dual, rows, k))
        return set_error(ARC_E_UNSUPPORTED_SHAPE, "matvec_imma: shape outside K/256 <= 14 (even for Q6_K)");
    if (!w0 || !x || !y || (dual && !w1)) return set_error(ARC_E_INVALID_ARGUMENT, "matvec: null pointer");
    if ((reinterpret_cast<uintptr_t>(w0) & 15u) || (w1 && (reinterpret_cast<uintptr_t>(w1) & 15u)))
        return set_error(ARC_E_ALIGNMENT, "matvec: weight pointers must be 16-byte aligned");
    int st = matvec_imma_prepare();
    if (st != ARC_OK) return st;
    const ImmaConfig c = imma_config(fmt, dual, k);
    const uint32_t nb = k / 256u;
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
    p.rb = nb * (fmt == 12 ? 144u : 210u);
    p.G = c.G;
    p.n_groups = (rows + c.G - 1u) / c.G;
    p.stages = c.S;
    p.stage_smem = c.stage_smem;
    p.x_floats = 0;
    static int sm_count[64] = {};  // per device, queried once
    int dev = 0;
    cudaGetDevice(&dev);
    int& sms = sm_count[dev & 63];
    if (sms <= 0 && cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) sms = 148;
    const uint32_t grid = std::min(p.n_groups, (uint32_t)sms);
    cudaError_t e;
    if (fmt == 12) {
        if (dual)
            e = c.MT == 2 ? launch_imma_t<12, 2, true>(p, nb, c.smem, grid, stream)
                          : launch_imma_t<12, 1, true>(p, nb, c.smem, grid, stream);
        else
            e = c.MT == 2 ? launch_imma_t<12, 2, false>(p, nb, c.smem, grid, stream)
                          : launch_imma_t<12, 1, false>(p, nb, c.smem, grid, stream);
    } else {
        e = c.MT == 2 ? launch_imma_t<14, 2, false>(p, nb, c.smem, grid, stream)
                      : launch_imma_t<14, 1, false>(p, nb, c.smem, grid, stream);
    }
    if (e != cudaSuccess) return set_cuda_error(e, "matvec_imma launch");
    return ARC_OK;
}

}  // namespace arc
