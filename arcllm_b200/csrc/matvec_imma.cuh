// Device pieces shared by the integer-MMA matvec kernels (matvec_imma.cu:
// whole-row stages for K <= 3584; matvec_imma_splitk.cu: K-chunked stages
// with a cross-CTA reduction): the MMA wrapper, the activation quantiser
// (22-bit block fixed point in three int8 limbs), the routed B-fragment
// gather, and the per-tile Q4_K / Q6_K multiply-accumulate + scale epilogue.
#pragma once
#include <cstdint>

#include "common.cuh"

namespace arc {
namespace {

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

// Two fp32 lanes per instruction (fma.rn.f32x2 / mul.rn.f32x2): each lane is
// rounded exactly as the scalar fmaf / __fmul_rn would round it.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 a, b, c;\n\t"
        "mov.b64 a, {%2, %3};\n\t"
        "mov.b64 b, {%4, %5};\n\t"
        "mov.b64 c, {%6, %7};\n\t"
        "fma.rn.f32x2 c, a, b, c;\n\t"
        "mov.b64 {%0, %1}, c;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 a, b, c;\n\t"
        "mov.b64 a, {%2, %3};\n\t"
        "mov.b64 b, {%4, %5};\n\t"
        "mul.rn.f32x2 c, a, b;\n\t"
        "mov.b64 {%0, %1}, c;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
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

// Quantise 256 activations (8 windows of 32) into limb planes and window
// constants.  Lane L holds elements 8(L&3)..+7 of window L>>2 in v[] (already
// RMS-normalised when that is fused).  planes: [3][256] int8 limbs l0, l1, l2
// (x_int = 65536 l0 + 256 l1 + l2); kc: [8][6] per window: 2^e (NaN if the
// window holds a non-finite value), sum of x (Q4_K dmin term), and for each
// 16-element half 32*... integer limb sums (Q6_K -32 offset term).
template <int FMT>
__device__ __forceinline__ void quantize8(const float (&v)[8], uint32_t lane, uint8_t* planes, float* kc) {
    const uint32_t jw = lane >> 2, qd = lane & 3u;  // window, quarter of the window
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
    *reinterpret_cast<uint2*>(planes + o) =
        make_uint2(pack4(l0[0], l0[1], l0[2], l0[3]), pack4(l0[4], l0[5], l0[6], l0[7]));
    *reinterpret_cast<uint2*>(planes + 256 + o) =
        make_uint2(pack4(l1[0], l1[1], l1[2], l1[3]), pack4(l1[4], l1[5], l1[6], l1[7]));
    *reinterpret_cast<uint2*>(planes + 512 + o) =
        make_uint2(pack4(l2[0], l2[1], l2[2], l2[3]), pack4(l2[4], l2[5], l2[6], l2[7]));
    if (FMT != 14) {  // Q4_K and EXEC148: one scale per 32-element window
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
}

// This lane's routed B fragments and epilogue constants for one 256-element
// slice whose windows 0..3 come from (pA, kA) and 4..7 from (pB, kB) -- the
// same set twice for a whole super-block, two blocks' halves for the Q6_K
// half-block pairing.
template <int FMT>
__device__ __forceinline__ void gather_xfrag(const uint8_t* pA, const float* kA, const uint8_t* pB, const float* kB,
                                             uint32_t lane, XFrag& f) {
    const uint32_t g = lane >> 2, t = lane & 3u, c = g >> 1, L = g & 1u;
    if (FMT == 12) {
        // window m = sub-block s; slots 4t..4t+3 <- elements 8t..8t+3, slots 16+4t.. <- 8t+4..8t+7.
        // This lane's nonzero windows are s = c (from A) and c + 4 (from B).
        uint2 w1[2], w2[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint8_t* pl = h ? pB : pA;
            const uint32_t off = 32u * (c + 4u * h) + 8u * t;
            w1[h] = *reinterpret_cast<const uint2*>(pl + 256u * L + off);
            w2[h] = L == 0 ? *reinterpret_cast<const uint2*>(pl + 512u + off) : make_uint2(0u, 0u);
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
            const float* kc = i ? kB : kA;
            const uint32_t sb = 4u * i + t;
            f.sx[i] = kc[6 * sb] * hi;
            f.xs[i] = kc[6 * sb + 1];
        }
        f.sx[2] = f.sx[3] = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) f.xh[i] = f.xl[i] = 0;
    } else {
        // window m = 4h + q (quarter q of half h); slot k <- element l = k; groups lh = k >> 4.
        // This lane's nonzero words: windows m with (q & 1) == c >> 1, i.e. q = (c >> 1) + {0, 2},
        // register b0 (l = 4t..) when c is even, b1 (l = 16 + 4t..) when c is odd.
        const uint32_t qlo = c >> 1, lh = c & 1u;
        uint32_t w1[2][2], w2[2][2];  // [h][q = qlo + 2i]
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint8_t* pl = h ? pB : pA;
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const uint32_t off = 32u * (4u * h + qlo + 2u * i) + 16u * lh + 4u * t;
                w1[h][i] = *reinterpret_cast<const uint32_t*>(pl + 256u * L + off);
                w2[h][i] = L == 0 ? *reinterpret_cast<const uint32_t*>(pl + 512u + off) : 0u;
            }
        }
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            const int h = m >> 2, q = m & 3;
            const bool on = (uint32_t)(q & 1) == qlo;
            const uint32_t v1 = on ? w1[h][q >> 1] : 0u, v2 = on ? w2[h][q >> 1] : 0u;
            f.b1[m][0] = lh == 0 ? v1 : 0u;
            f.b1[m][1] = lh == 1 ? v1 : 0u;
            f.b2[m][0] = lh == 0 ? v2 : 0u;
            f.b2[m][1] = lh == 1 ? v2 : 0u;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float* kc = (i >> 1) ? kB : kA;
            const uint32_t j = 4u * (i >> 1) + 2u * (i & 1) + (t >> 1), lh = t & 1u;
            f.sx[i] = kc[6 * j];
            f.xh[i] = 32 * __float_as_int(kc[6 * j + 2 + 2 * lh]);
            f.xl[i] = 32 * __float_as_int(kc[6 * j + 3 + 2 * lh]);
        }
        f.xs[0] = f.xs[1] = 0.f;
    }
}

// Routed B fragments for the EXEC148 layout (148-byte blocks: d, dmin, eight
// (sc, mn) bytes, then window j's 32 codes as 16 bytes of element pairs,
// byte b = q[2b] | q[2b+1] << 4).  MMA m = 2p + hh of a block takes the 32
// code bytes of windows 2p, 2p+1: k slot 4u+i <- byte 8u+i, slot 16+4u+i <-
// byte 8u+4+i, low nibbles (hh = 0: even elements) or high nibbles shifted
// down (hh = 1: odd elements).  Byte b of that span is byte b & 15 of window
// 2p + (b >> 4), so lane (g, t) (column pair c = g >> 1, limb g & 1) carries
// window w = 2p + (t >> 1) -- elements 16(t&1) + hh + 2i (b0) and
// 16(t&1) + 8 + hh + 2i (b1), i = 0..3 -- when w & 3 == c, zeros otherwise.
// Windows 4i .. 4i+3 accumulate in D[i], so lane t applies the scales of
// windows t and 4 + t, as for Q4_K.
__device__ __forceinline__ void gather_xfrag_e148(const uint8_t* pl, const float* kc, uint32_t lane, XFrag& f) {
    const uint32_t g = lane >> 2, t = lane & 3u, c = g >> 1, L = g & 1u;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const uint32_t w = 2u * p + (t >> 1);
        const bool on = (w & 3u) == c;
        const uint4 q1 = *reinterpret_cast<const uint4*>(pl + 256u * L + 32u * w + 16u * (t & 1u));
        const uint4 q2 = L == 0 ? *reinterpret_cast<const uint4*>(pl + 512u + 32u * w + 16u * (t & 1u))
                                : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const uint32_t sel = hh ? 0x7531u : 0x6420u;  // odd or even bytes of a word pair
            const int m = 2 * p + hh;
            f.b1[m][0] = on ? __byte_perm(q1.x, q1.y, sel) : 0u;
            f.b1[m][1] = on ? __byte_perm(q1.z, q1.w, sel) : 0u;
            f.b2[m][0] = on ? __byte_perm(q2.x, q2.y, sel) : 0u;
            f.b2[m][1] = on ? __byte_perm(q2.z, q2.w, sel) : 0u;
        }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const uint32_t w = 4u * i + t;
        f.sx[i] = kc[6 * w];
        f.xs[i] = kc[6 * w + 1];
    }
    f.sx[2] = f.sx[3] = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) f.xh[i] = f.xl[i] = 0;
}

// One 16-row tile x one EXEC148 block (row offsets r0, r1 of the block in the
// stage, 4-byte aligned): adds the rows' partial dot products (windows t and
// 4 + t of this lane) to y0 and y1.  w = d*sc*q - dmin*mn as for Q4_K
// (shaders/q4_down_exec148_serial.comp:6 computes the same per element).
__device__ __forceinline__ void e148_tile(const uint8_t* st, uint32_t r0, uint32_t r1, uint32_t t, const XFrag& f,
                                          float& y0, float& y1) {
    constexpr uint32_t K = 0x0F0F0F0Fu;
    int D1[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}}, D2[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const uint32_t o = 20u + 32u * p + 8u * t;
        const uint32_t a0 = *reinterpret_cast<const uint32_t*>(st + r0 + o);
        const uint32_t a2 = *reinterpret_cast<const uint32_t*>(st + r0 + o + 4u);
        const uint32_t a1 = *reinterpret_cast<const uint32_t*>(st + r1 + o);
        const uint32_t a3 = *reinterpret_cast<const uint32_t*>(st + r1 + o + 4u);
        const int i = p >> 1;
        imma(D1[i], a0 & K, a1 & K, a2 & K, a3 & K, f.b1[2 * p][0], f.b1[2 * p][1]);
        imma(D2[i], a0 & K, a1 & K, a2 & K, a3 & K, f.b2[2 * p][0], f.b2[2 * p][1]);
        imma(D1[i], (a0 >> 4) & K, (a1 >> 4) & K, (a2 >> 4) & K, (a3 >> 4) & K, f.b1[2 * p + 1][0],
             f.b1[2 * p + 1][1]);
        imma(D2[i], (a0 >> 4) & K, (a1 >> 4) & K, (a2 >> 4) & K, (a3 >> 4) & K, f.b2[2 * p + 1][0],
             f.b2[2 * p + 1][1]);
    }
    float out[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const uint8_t* blk = st + (r ? r1 : r0);
        const uint32_t hd = *reinterpret_cast<const uint32_t*>(blk);
        const float d = __half2float(__ushort_as_half((unsigned short)(hd & 0xffffu)));
        const float dmin = __half2float(__ushort_as_half((unsigned short)(hd >> 16)));
        const uint32_t s0 = *reinterpret_cast<const unsigned short*>(blk + 4u + 2u * t);   // (sc, mn) of window t
        const uint32_t s1 = *reinterpret_cast<const unsigned short*>(blk + 12u + 2u * t);  // window 4 + t
        const float F0 = combine(D1[0][2 * r], D1[0][2 * r + 1], D2[0][2 * r], 0, 0);
        const float F1 = combine(D1[1][2 * r], D1[1][2 * r + 1], D2[1][2 * r], 0, 0);
        const float tt = fmaf((float)(s0 & 255u) * f.sx[0], F0, ((float)(s1 & 255u) * f.sx[1]) * F1);
        const float uu = fmaf((float)(s0 >> 8), f.xs[0], (float)(s1 >> 8) * f.xs[1]);
        out[r] = fmaf(d, tt, -dmin * uu);
    }
    y0 += out[0];
    y1 += out[1];
}

// The four 4-code words of one (ql word a, ql word b = a + 32 bytes, qh word)
// triple: code = low or high nibble | two qh bits << 4.  qh is split once into
// the bit pairs of quarters 0/2 (0x33) and 1/3 (0xCC), so each code word is one
// shift and one bit-select (the other bit positions of the shifted pair are
// zero or fall in the nibble half of the select).
__device__ __forceinline__ void q6_codes(uint32_t a, uint32_t b, uint32_t qh, uint32_t (&v)[4]) {
    constexpr uint32_t K = 0x0F0F0F0Fu;
    const uint32_t qm = qh & 0x33333333u, qn = qh & 0xCCCCCCCCu;
    v[0] = (a & K) | ((qm << 4) & ~K);
    v[1] = (b & K) | ((qn << 2) & ~K);
    v[2] = ((a >> 4) & K) | (qm & ~K);
    v[3] = ((b >> 4) & K) | ((qn >> 2) & ~K);
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
// The two MMAs into one accumulator are issued apart (window order 0, 2, 1, 3)
// and the scale epilogue runs on both rows at once in packed fp32 pairs (the
// same roundings per row as the scalar form).
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
                q6_codes(qa, qb, qh, v[lh][r]);
            }
        }
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
            const int q = ((qq & 1) << 1) | (qq >> 1);
            const int m = 4 * h + q, i = 2 * h + (q >> 1);
            imma(D1[i], v[0][0][q], v[0][1][q], v[1][0][q], v[1][1][q], f.b1[m][0], f.b1[m][1]);
            imma(D2[i], v[0][0][q], v[0][1][q], v[1][0][q], v[1][1][q], f.b2[m][0], f.b2[m][1]);
        }
    }
    float2 part[2];  // [half] (row0, row1)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int8_t* sc0 = reinterpret_cast<const int8_t*>(st + row0 + (h ? offB : offA) + 192u + t);
        const int8_t* sc1 = reinterpret_cast<const int8_t*>(st + row1 + (h ? offB : offA) + 192u + t);
        float2 acc = make_float2(0.f, 0.f);
#pragma unroll
        for (int ii = 0; ii < 2; ++ii) {
            const int i = 2 * h + ii;
            const float2 hi = make_float2((float)(D1[i][0] * 256 + D1[i][1] - f.xh[i]),
                                          (float)(D1[i][2] * 256 + D1[i][3] - f.xh[i]));
            const float2 lo = make_float2((float)(D2[i][0] - f.xl[i]), (float)(D2[i][2] - f.xl[i]));
            const float2 F = fma2(hi, make_float2(256.0f, 256.0f), lo);
            const float2 s = mul2(make_float2((float)sc0[4 * i], (float)sc1[4 * i]), make_float2(f.sx[i], f.sx[i]));
            acc = fma2(s, F, acc);
        }
        part[h] = acc;
    }
    auto d_of = [&](uint32_t ro, uint32_t off) {
        return __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(st + ro + off + 208u)));
    };
    const float2 dA = make_float2(d_of(row0, offA), d_of(row1, offA));
    const float2 dB = make_float2(d_of(row0, offB), d_of(row1, offB));
    const float2 o = fma2(dA, part[0], mul2(dB, part[1]));
    y0 += o.x;
    y1 += o.y;
}

// q6_tile with each half's scale epilogue run right after its MMAs, so only
// half the accumulators are live at a time (for kernels with more state of
// their own in registers).  Same arithmetic, same order of fp32 operations.
template <bool ODD0>
__device__ __forceinline__ void q6_tile_lowreg(const uint8_t* st, uint32_t row0, uint32_t row1, uint32_t offA,
                                               uint32_t offB, uint32_t t, const XFrag& f, float& y0, float& y1) {
    float part[2][2];  // [row][half]
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const bool odd = (h == 0) ? ODD0 : !ODD0;
        const uint32_t boff = h ? offB : offA;
        int D1[2][4], D2[2][4];
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) D1[i][j] = D2[i][j] = 0;
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
                q6_codes(qa, qb, qh, v[lh][r]);
            }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int m = 4 * h + q, ii = q >> 1;
            imma(D1[ii], v[0][0][q], v[0][1][q], v[1][0][q], v[1][1][q], f.b1[m][0], f.b1[m][1]);
            imma(D2[ii], v[0][0][q], v[0][1][q], v[1][0][q], v[1][1][q], f.b2[m][0], f.b2[m][1]);
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const uint32_t ro = r ? row1 : row0;
            const int8_t* sc = reinterpret_cast<const int8_t*>(st + ro + boff + 192u + t);
            float acc = 0.f;
#pragma unroll
            for (int ii = 0; ii < 2; ++ii) {
                const int i = 2 * h + ii;
                const float F = combine(D1[ii][2 * r], D1[ii][2 * r + 1], D2[ii][2 * r], f.xh[i], f.xl[i]);
                acc = fmaf((float)sc[4 * i] * f.sx[i], F, acc);
            }
            part[r][h] = acc;
        }
    }
    float out[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const uint32_t ro = r ? row1 : row0;
        const float dA = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(st + ro + offA + 208u)));
        const float dB = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(st + ro + offB + 208u)));
        out[r] = fmaf(dA, part[r][0], dB * part[r][1]);
    }
    y0 += out[0];
    y1 += out[1];
}

// Whole-row kernels: the warp's x slice (windows 0..3 from block bA, 4..7 from block bB):
// load, fuse the RMSNorm (sum of squares over all warps, in double), quantise
// into the warp's scratch, gather this lane's fragments.
template <int FMT>
__device__ __forceinline__ void build_xfrag(const float* x, const float* gamma, float eps, uint32_t k, double* red_d,
                                            uint32_t nwc, uint32_t warp, uint32_t bA, uint32_t bB, uint32_t lane,
                                            uint8_t* xs, XFrag& f) {
    const uint32_t jw = lane >> 2, qd = lane & 3u;
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
    float* kc = reinterpret_cast<float*>(xs + 768);
    quantize8<FMT>(v, lane, xs, kc);
    __syncwarp();
    gather_xfrag<FMT>(xs, kc, xs, kc, lane, f);
}

}  // namespace
}  // namespace arc
