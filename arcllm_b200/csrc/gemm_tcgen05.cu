// Prefill GEMM on the 5th-generation tensor cores: Y[M x N] (fp32) =
// X[M x K] (bf16) * W^T with W the N x K Q4_K matrix of a projection, M <= 256
// prompt tokens.  The counterpart of the reference's prefill kernels
// (shaders/p7l_ffn_q4k_gateup_fused.comp, shaders/p7g_ffn_q4k_tiled16.comp:
// weights dequantised into shared memory, then a tiled multiply), rebuilt for
// sm_100a with tcgen05.mma, TMEM accumulators and TMA.
//
// One CTA computes all M (<= 256) rows x 128 columns of Y:
//   warp 0      TMA producer: two 128-row boxes of X per 64-wide K step
//               (128-byte swizzle, the UMMA K-major SW128 layout);
//   warp 1      allocates 256 TMEM columns (two 128x128 fp32 accumulators)
//               and issues tcgen05.mma (M=128, N=128, K=16, bf16 x bf16 -> f32)
//               from one thread, committing each stage back to its "empty"
//               barrier;
//   warps 2..9  dequantise the 128 W rows x 64 K of each stage from Q4_K to
//               bf16 straight into the swizzled layout (one 32-weight
//               sub-block per thread, packed bytes prefetched 4 stages
//               ahead), then read the accumulators back with tcgen05.ld
//               (warp w serves TMEM lanes 32*(w%4)..) and store Y.
// Both MMAs of a K step share the dequantised B tile, so each weight is
// dequantised once per CTA.  The operands are bf16, fp16 (same rate, 11
// instead of 8 significant bits), or fp16 hi + lo pairs of both X and W with
// three MMAs per K step (~22 bits: the projections whose outputs feed the
// attention scores).  When N/128 tiles leave SMs idle (the FFN-down
// shape, N = 3584), K is split across CTAs, the CTAs store partial tiles and
// a grid-wide reduce kernel adds them in split order (deterministic; the
// last CTA of each column tile adding them alone was the slowest part of the
// small-N GEMMs).  All waits are bounded; on a timeout the kernel
// sets the device error word, lets in-flight copies and MMAs finish (bounded),
// frees its TMEM and returns.
#include <cuda.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <mutex>

#include "arcllm_cuda_internal.h"
#include "common.cuh"

namespace arc {
namespace {

constexpr uint32_t kBN = 128;          // output columns per CTA
constexpr uint32_t kBK = 64;           // K per stage (128 bytes of bf16: one swizzle row)
constexpr uint32_t kAHalf = 128 * kBK * 2;   // 16 KB: one 128-row box of X
constexpr uint32_t kBTile = kBN * kBK * 2;   // 16 KB: dequantised W tile
constexpr uint32_t kDqWarps = 8;                         // dequantising warps: 2 threads per W row
constexpr uint32_t kThreads = (2 + kDqWarps) * 32;
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kMaxStages = 4;

// Operand modes: bf16 (0), fp16 (1), fp16 x3 (2): X = X_hi + X_lo and
// W = W_hi + W_lo as fp16 pairs (W_hi = fp16(w), W_lo = fp16(w - W_hi) of the
// exactly dequantised fp32 weight), accumulated as X_hi W_hi + X_lo W_hi +
// X_hi W_lo -- ~22 significant bits of each operand, at three MMAs per K step.
// Modes 0/1 stage two 128-row boxes of X and one W tile (48 KB, 4 stages);
// mode 2 four boxes (hi and lo) and two W tiles (96 KB, 2 stages).
template <int MODE>
struct GemmStage {
    static constexpr uint32_t kABoxes = MODE == 2 ? 4u : 2u;
    static constexpr uint32_t kBTiles = MODE == 2 ? 2u : 1u;
    static constexpr uint32_t kStages = MODE == 2 ? 2u : 4u;
    static constexpr uint32_t kBOff = kABoxes * kAHalf;
    static constexpr uint32_t kBytes = kBOff + kBTiles * kBTile;
};

struct GemmSmemTail {
    uint64_t full_a[kMaxStages];
    uint64_t full_b[kMaxStages];
    uint64_t empty[kMaxStages];
    uint64_t done;
    uint32_t tmem_base;
    int abort_flag;
};

// Split-K: CTAs (tile, split) cover K super-blocks [nsb*split/ks, nsb*(split+1)/ks)
// and store their partial tiles to ws[split][m][n]; a grid-wide reduce kernel
// then adds them in split order (deterministic) plus the residual into y.
struct SplitKWs {
    float* ws;
    uint32_t ks;
};

template <int MODE>
constexpr uint32_t smem_bytes() {  // + alignment slack
    return GemmStage<MODE>::kStages * GemmStage<MODE>::kBytes + (uint32_t)sizeof(GemmSmemTail) + 1024u;
}
static_assert(smem_bytes<0>() <= 232448u && smem_bytes<2>() <= 232448u, "GEMM stages exceed 227 KB");

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// UMMA shared-memory descriptor for a K-major tile in the 128-byte swizzle
// layout: 8-row x 128-byte atoms stacked along M/N (stride 1024 bytes).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);        // start address / 16
    d |= (uint64_t)1u << 16;                         // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024u >> 4) << 32;               // stride byte offset: 8 rows x 128 B
    d |= (uint64_t)1u << 46;                         // descriptor version (sm_100)
    d |= (uint64_t)2u << 61;                         // layout: 128-byte swizzle
    return d;
}

// kind::f16 instruction descriptor: A and B both bf16 (F16 = false) or both fp16
// (F16 = true), K-major, f32 accumulator, M=128, N=128
template <bool F16>
constexpr uint32_t idesc() {
    return (1u << 4)                  // D format f32
           | ((F16 ? 0u : 1u) << 7)   // A format: 0 f16, 1 bf16
           | ((F16 ? 0u : 1u) << 10)  // B format: 0 f16, 1 bf16
           | ((kBN >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        :
        : "r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

template <bool F16>
__device__ __forceinline__ void umma_16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        :
        : "r"(tmem_d), "l"(da), "l"(db), "r"(idesc<F16>()), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

__device__ __forceinline__ uint32_t f16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// Packed 16-bit pairs of the GEMM's operand type: bf16 (F16 = false) or fp16.
template <bool F16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    return F16 ? f16x2(lo, hi) : bf16x2(lo, hi);
}
// x2 arithmetic on raw bits (both halves), one rounding each
template <bool F16>
__device__ __forceinline__ uint32_t sub2(uint32_t a, uint32_t b) {
    uint32_t r;
    if (F16)
        asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    else
        asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
template <bool F16>
__device__ __forceinline__ uint32_t fma2(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    if (F16)
        asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    else
        asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}
// x2 of the value B with small integers c exact as (B + c) - B: the bit
// pattern of B ORed with c (B = 128 in bf16, 1024 in fp16: ulp 1 there)
template <bool F16>
constexpr uint32_t kIntBase2 = F16 ? 0x64006400u : 0x43004300u;
// x2 of B + 32 (the Q6_K code offset folded into the subtraction)
template <bool F16>
constexpr uint32_t kIntBase32x2 = F16 ? 0x64206420u : 0x43204320u;

// Per super-block constants of one thread's sub-blocks 2c + hi (c = 0..3):
// scale f = d*sc and offset -(dmin*mn), each rounded to the operand type and
// broadcast to both halves of a pair.  src/p8c_segmented_access_correctness.cpp:531-540
// (scale/min unpacking), :1166-1181 (w = d*sc*q - dmin*mn).
template <bool F16>
__device__ __forceinline__ void subblock_consts(uint4 hd, uint32_t hi, uint32_t (&fb)[4], uint32_t (&ob)[4]) {
    const uint32_t S[3] = {hd.y, hd.z, hd.w};
    auto sbyte = [&](uint32_t i) { return (S[i >> 2] >> (8u * (i & 3u))) & 0xFFu; };
    const float d = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xFFFFu)));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
#pragma unroll
    for (uint32_t c = 0; c < 4; ++c) {
        const uint32_t j = 2u * c + hi;
        uint32_t sc, mn;
        if (j < 4) {
            sc = sbyte(j) & 63u;
            mn = sbyte(j + 4) & 63u;
        } else {
            sc = (sbyte(j + 4) & 15u) | ((sbyte(j - 4) >> 6) << 4);
            mn = (sbyte(j + 4) >> 4) | ((sbyte(j) >> 6) << 4);
        }
        fb[c] = pack2<F16>(d * (float)sc, d * (float)sc);
        ob[c] = pack2<F16>(-(dmin * (float)mn), -(dmin * (float)mn));
    }
}

// Dequantise the 32 weights of sub-block 2c+hi of one Q4_K row -- elements
// 32*hi .. +31 of the 64-element stage row, the low (hi=0) or high (hi=1)
// nibbles of its 32 code bytes -- to bf16 (fp16) pairs: q via (B + q) - B
// (exact; B = 128 in bf16, 1024 in fp16), then one x2 FMA q*f - o (one
// rounding).  Stored as 16-byte chunks 4*hi .. 4*hi+3 of row n of the
// swizzled B tile.
template <bool F16>
__device__ __forceinline__ void dequant_subblock(uint4 q0, uint4 q1, uint32_t fb, uint32_t ob, uint32_t n, uint32_t hi,
                                                 uint8_t* btile) {
    const uint32_t w8[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    uint8_t* rowbase = btile + (n >> 3) * 1024u + (n & 7u) * 128u;
    constexpr uint32_t k128 = kIntBase2<F16>;
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {  // output chunk: elements 8*ch .. +7 = code bytes 8*ch .. +7
        uint32_t out[4];
#pragma unroll
        for (int pr = 0; pr < 4; ++pr) {
            const uint32_t word = w8[2 * ch + (pr >> 1)];
            // bytes (2*(pr&1), 2*(pr&1)+1) of the word into the low byte of each 16-bit half
            const uint32_t spread = __byte_perm(word, 0u, (pr & 1) ? 0x4342u : 0x4140u);
            const uint32_t q = hi ? ((spread >> 4) & 0x000F000Fu) : (spread & 0x000F000Fu);
            out[pr] = fma2<F16>(sub2<F16>(q | k128, k128), fb, ob);
        }
        const uint32_t chunk = 4u * hi + ch;
        *reinterpret_cast<uint4*>(rowbase + ((chunk ^ (n & 7u)) << 4)) = make_uint4(out[0], out[1], out[2], out[3]);
    }
}

// 8 little-endian words of the 32 bytes at a 2-byte-aligned global address,
// from 9 aligned word loads (the word past the end stays inside the Q6_K
// block for every caller) and funnel shifts.
struct Raw9 {
    uint32_t r[9];
};
__device__ __forceinline__ void ld_raw9(const uint8_t* p, Raw9& o) {
    const uint32_t* a = reinterpret_cast<const uint32_t*>(reinterpret_cast<uintptr_t>(p) & ~uintptr_t(3));
#pragma unroll
    for (int i = 0; i < 9; ++i) o.r[i] = __ldg(a + i);
}
__device__ __forceinline__ uint32_t raw9_word(const Raw9& o, int i, uint32_t sh) {
    return __funnelshift_r(o.r[i], o.r[i + 1], sh);
}

// Dequantise quarter q of half h of one Q6_K super-block row -- 32 weights,
// elements 32*hi .. +31 of the 64-element stage row -- to bf16 (fp16): the
// 6-bit code c = low nibble of ql | 2 bits of qh << 4
// (src/p8c_segmented_access_correctness.cpp:905-956), c - 32 via (B + c) - (B + 32)
// (exact), times f = d * sc rounded to the operand type, with one rounding;
// scales sc[8h + 2q] (elements 0..15) and sc[8h + 2q + 1] (16..31).
template <bool F16>
__device__ __forceinline__ void dequant_q6_quarter(const Raw9& ql, uint32_t shl, const Raw9& qh, uint32_t shh,
                                                   uint32_t lo_shift, uint32_t qh_shift, uint32_t f0, uint32_t f1,
                                                   uint32_t n, uint32_t hi, uint8_t* btile) {
    uint8_t* rowbase = btile + (n >> 3) * 1024u + (n & 7u) * 128u;
    constexpr uint32_t k128 = kIntBase2<F16>, k160 = kIntBase32x2<F16>, kNegZero = 0x80008000u;
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {  // output chunk: elements 8*ch .. +7
        uint32_t out[4];
#pragma unroll
        for (int wi = 0; wi < 2; ++wi) {
            const int i = 2 * ch + wi;
            const uint32_t c = ((raw9_word(ql, i, shl) >> lo_shift) & 0x0F0F0F0Fu) |
                               (((raw9_word(qh, i, shh) >> qh_shift) & 0x03030303u) << 4);
#pragma unroll
            for (int pr = 0; pr < 2; ++pr) {
                const uint32_t spread = __byte_perm(c, 0u, pr ? 0x4342u : 0x4140u);
                out[2 * wi + pr] = fma2<F16>(sub2<F16>(spread | k128, k160), ch < 2 ? f0 : f1, kNegZero);
            }
        }
        const uint32_t chunk = 4u * hi + ch;
        *reinterpret_cast<uint4*>(rowbase + ((chunk ^ (n & 7u)) << 4)) = make_uint4(out[0], out[1], out[2], out[3]);
    }
}

// Mode 2: the fp16 hi / lo halves of 8 fp32 weights (elements 8*chunk .. +7
// of row n of the stage) into the W_hi and W_lo tiles (same swizzled place).
__device__ __forceinline__ void store_hi_lo8(const float (&w)[8], uint32_t n, uint32_t chunk, uint8_t* bh,
                                             uint8_t* bl) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        h[i] = f16x2(w[2 * i], w[2 * i + 1]);
        const float2 hf = __half22float2(*reinterpret_cast<const __half2*>(&h[i]));
        l[i] = f16x2(w[2 * i] - hf.x, w[2 * i + 1] - hf.y);  // w - hi is exact in fp32
    }
    const uint32_t off = (n >> 3) * 1024u + (n & 7u) * 128u + ((chunk ^ (n & 7u)) << 4);
    *reinterpret_cast<uint4*>(bh + off) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(bl + off) = make_uint4(l[0], l[1], l[2], l[3]);
}

// Mode 2, Q4_K: the per-sub-block scale f = d*sc and offset o = -(dmin*mn)
// in fp32 (both exact: fp16 times a 6-bit integer) for sub-blocks 2c + hi.
__device__ __forceinline__ void subblock_consts_f32(uint4 hd, uint32_t hi, float (&f)[4], float (&o)[4]) {
    const uint32_t S[3] = {hd.y, hd.z, hd.w};
    auto sbyte = [&](uint32_t i) { return (S[i >> 2] >> (8u * (i & 3u))) & 0xFFu; };
    const float d = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xFFFFu)));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
#pragma unroll
    for (uint32_t c = 0; c < 4; ++c) {
        const uint32_t j = 2u * c + hi;
        uint32_t sc, mn;
        if (j < 4) {
            sc = sbyte(j) & 63u;
            mn = sbyte(j + 4) & 63u;
        } else {
            sc = (sbyte(j + 4) & 15u) | ((sbyte(j - 4) >> 6) << 4);
            mn = (sbyte(j + 4) >> 4) | ((sbyte(j) >> 6) << 4);
        }
        f[c] = d * (float)sc;
        o[c] = -(dmin * (float)mn);
    }
}

// Mode 2, Q4_K: the 32 weights of sub-block 2c + hi as fp32 exactly as the
// reference dequantises them (f*q is exact, so fmaf(f, q, o) rounds once like
// (d*sc)*q - dmin*mn, src/p8c_segmented_access_correctness.cpp:1166-1181),
// split into fp16 hi / lo tiles.
__device__ __forceinline__ void dequant_subblock_x3(uint4 q0, uint4 q1, float f, float o, uint32_t n, uint32_t hi,
                                                    uint8_t* bh, uint8_t* bl) {
    const uint32_t w8[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
        float w[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t byte = (w8[2 * ch + (j >> 2)] >> (8 * (j & 3))) & 0xFFu;
            const uint32_t q = hi ? (byte >> 4) : (byte & 15u);
            w[j] = fmaf(f, (float)q, o);
        }
        store_hi_lo8(w, n, 4u * hi + ch, bh, bl);
    }
}

// Mode 2, Q6_K: quarter q of half h of a super-block row (see dequant_q6_quarter),
// w = (d*sc) * (c - 32) in fp32 (src/p8c_segmented_access_correctness.cpp:944-956),
// split into fp16 hi / lo tiles.
__device__ __forceinline__ void dequant_q6_quarter_x3(const Raw9& ql, uint32_t shl, const Raw9& qh, uint32_t shh,
                                                      uint32_t lo_shift, uint32_t qh_shift, float f0, float f1,
                                                      uint32_t n, uint32_t hi, uint8_t* bh, uint8_t* bl) {
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
        float w[8];
#pragma unroll
        for (int wi = 0; wi < 2; ++wi) {
            const int i = 2 * ch + wi;
            const uint32_t c4 = ((raw9_word(ql, i, shl) >> lo_shift) & 0x0F0F0F0Fu) |
                                (((raw9_word(qh, i, shh) >> qh_shift) & 0x03030303u) << 4);
#pragma unroll
            for (int b = 0; b < 4; ++b)
                w[4 * wi + b] = __fmul_rn(ch < 2 ? f0 : f1, (float)((int)((c4 >> (8 * b)) & 0xFFu) - 32));
        }
        store_hi_lo8(w, n, 4u * hi + ch, bh, bl);
    }
}

// MODE 0: bf16 operands; 1: fp16 (11 significant bits instead of 8: the
// scale and offset of each sub-block, q*f - o and X all round 8x more finely,
// at the same tensor-core rate); 2: fp16 hi + lo of both operands, three MMAs
// per K step (xmap_lo: the X_lo tensor).
template <int FMT, int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kq_bf16_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap xmap_lo,
                        const uint8_t* __restrict__ w, uint32_t n_total, uint32_t k, uint32_t m,
                        const float* __restrict__ residual, float* __restrict__ y, unsigned int* err,
                        const SplitKWs sk) {
    pdl_wait();  // X and the residual may come from the preceding kernels (a no-op for a plain launch)
    constexpr bool F16 = MODE >= 1;
    constexpr uint32_t kStages = GemmStage<MODE>::kStages, kStageBytes = GemmStage<MODE>::kBytes;
    constexpr uint32_t kBOff = GemmStage<MODE>::kBOff;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_align_up<1024>(smem_raw, 0);
    GemmSmemTail* tail = reinterpret_cast<GemmSmemTail*>(smem + kStages * kStageBytes);
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    const uint32_t n0 = blockIdx.x * kBN;
    const uint32_t nsb = k / 256u, split = blockIdx.y;
    const uint32_t sb_begin = nsb * split / sk.ks, sb_end = nsb * (split + 1u) / sk.ks;
    const uint32_t kbase = 4u * sb_begin;          // first 64-wide K block of this CTA
    const uint32_t nkb = 4u * (sb_end - sb_begin);  // K blocks of this CTA
    constexpr uint32_t bsz = FMT == 12 ? 144u : 210u;
    const uint32_t rb = (k / 256u) * bsz;

    if (tid == 0) {
        for (uint32_t s = 0; s < kStages; ++s) {
            mbar_init(&tail->full_a[s], 1);
            mbar_init(&tail->full_b[s], kDqWarps);
            mbar_init(&tail->empty[s], 1);
        }
        mbar_init(&tail->done, 1);
        tail->abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {  // TMEM: two 128x128 fp32 accumulators
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tail->tmem_base)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = tail->tmem_base;
    volatile int* abort_flag = &tail->abort_flag;

    if (warp == 0) {
        // ---------------- TMA producer (X) ----------------
        uint32_t issued = 0;
        if (lane == 0) {
            for (uint32_t kb = 0; kb < nkb; ++kb) {
                const uint32_t s = kb % kStages;
                if (kb >= kStages && !mbar_wait(&tail->empty[s], ((kb / kStages) - 1u) & 1u, err)) {
                    *abort_flag = 1;
                    break;
                }
                if (*abort_flag) break;
                uint8_t* st = smem + s * kStageBytes;
                mbar_arrive_expect_tx(&tail->full_a[s], GemmStage<MODE>::kABoxes * kAHalf);
                tma_load_2d(smem_u32(st), &xmap, (int)((kbase + kb) * kBK), 0, &tail->full_a[s]);
                tma_load_2d(smem_u32(st + kAHalf), &xmap, (int)((kbase + kb) * kBK), 128, &tail->full_a[s]);
                if (MODE == 2) {  // boxes 2, 3: X_lo of the same rows
                    tma_load_2d(smem_u32(st + 2 * kAHalf), &xmap_lo, (int)((kbase + kb) * kBK), 0, &tail->full_a[s]);
                    tma_load_2d(smem_u32(st + 3 * kAHalf), &xmap_lo, (int)((kbase + kb) * kBK), 128,
                                &tail->full_a[s]);
                }
                ++issued;
            }
            if (*abort_flag)  // no copy may still be landing at exit
                for (uint32_t j = issued > kStages ? issued - kStages : 0; j < issued; ++j)
                    mbar_wait(&tail->full_a[j % kStages], (j / kStages) & 1u, err);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            for (uint32_t kb = 0; kb < nkb; ++kb) {
                const uint32_t s = kb % kStages, ph = (kb / kStages) & 1u;
                if (!mbar_wait(&tail->full_a[s], ph, err) || !mbar_wait(&tail->full_b[s], ph, err)) *abort_flag = 1;
                if (*abort_flag) break;
                asm volatile("tcgen05.fence::after_thread_sync;");
                const uint32_t st = smem_u32(smem + s * kStageBytes);
#pragma unroll
                for (uint32_t kk = 0; kk < kBK / 16u; ++kk) {
                    const uint64_t db = sw128_desc(st + kBOff + 32u * kk);
                    const uint32_t acc = (kb | kk) != 0u;
                    umma_16<F16>(tmem, sw128_desc(st + 32u * kk), db, acc);
                    umma_16<F16>(tmem + 128u, sw128_desc(st + kAHalf + 32u * kk), db, acc);
                    if (MODE == 2) {  // + X_lo W_hi + X_hi W_lo into the same accumulators
                        const uint64_t dbl = sw128_desc(st + kBOff + kBTile + 32u * kk);
                        umma_16<true>(tmem, sw128_desc(st + 2 * kAHalf + 32u * kk), db, 1u);
                        umma_16<true>(tmem + 128u, sw128_desc(st + 3 * kAHalf + 32u * kk), db, 1u);
                        umma_16<true>(tmem, sw128_desc(st + 32u * kk), dbl, 1u);
                        umma_16<true>(tmem + 128u, sw128_desc(st + kAHalf + 32u * kk), dbl, 1u);
                    }
                }
                umma_commit(&tail->empty[s]);  // stage free once these MMAs have read it
            }
            umma_commit(&tail->done);  // accumulators complete (also after an abort: drains issued MMAs)
        }
    } else {
        // ---------------- dequant producers, then epilogue ----------------
        const uint32_t dt = tid - 64u;  // 0..255: W row dt >> 1 of this CTA, sub-block half dt & 1 of the stage
        const uint32_t nrow = dt >> 1, hi = dt & 1u;
        const uint8_t* row = w + (uint64_t)(n0 + nrow) * rb + (uint64_t)sb_begin * bsz;  // this split's K range
        if (FMT == 14) {
            // Q6_K: thread (nrow, hi) dequantises quarter 2*(sub & 1) + hi of half sub >> 1 of each
            // super-block (sub = stage index within the super-block); raw words prefetched 2 stages ahead
            constexpr uint32_t kPf = 2;
            Raw9 pql[kPf], pqh[kPf];
            uint32_t psc[kPf];
            auto load6 = [&](uint32_t kb, Raw9& a, Raw9& b, uint32_t& scd) {
                const uint8_t* blk = row + (kb >> 2) * 210u;
                const uint32_t sub = kb & 3u, h = sub >> 1, q = 2u * (sub & 1u) + hi;
                ld_raw9(blk + 64u * h + 32u * hi, a);
                ld_raw9(blk + 128u + 32u * h, b);
                const uint32_t sc2 = *reinterpret_cast<const unsigned short*>(blk + 192u + 8u * h + 2u * q);
                const uint32_t dd = *reinterpret_cast<const unsigned short*>(blk + 208u);
                scd = sc2 | (dd << 16);
            };
#pragma unroll
            for (uint32_t i = 0; i < kPf; ++i)
                if (i < nkb) load6(i, pql[i], pqh[i], psc[i]);
            bool stop6 = false;
            for (uint32_t kb0 = 0; kb0 < nkb && !stop6; kb0 += kPf) {
#pragma unroll
              for (uint32_t slot = 0; slot < kPf; ++slot) {
                const uint32_t kb = kb0 + slot;
                if (kb >= nkb) break;
                const Raw9 ql = pql[slot], qh = pqh[slot];
                const uint32_t scd = psc[slot];
                const uint8_t* blk = row + (kb >> 2) * 210u;
                const uint32_t sub = kb & 3u, h = sub >> 1, q = 2u * (sub & 1u) + hi;
                const uint32_t shl = (uint32_t)((reinterpret_cast<uintptr_t>(blk + 64u * h + 32u * hi)) & 3u) * 8u;
                const uint32_t shh = (uint32_t)((reinterpret_cast<uintptr_t>(blk + 128u + 32u * h)) & 3u) * 8u;
                if (kb + kPf < nkb) load6(kb + kPf, pql[slot], pqh[slot], psc[slot]);
                const float d = __half2float(__ushort_as_half((unsigned short)(scd >> 16)));
                const float s0 = d * (float)(int8_t)(scd & 0xFFu), s1 = d * (float)(int8_t)((scd >> 8) & 0xFFu);
                const uint32_t f0 = pack2<F16 && MODE != 2>(s0, s0), f1 = pack2<F16 && MODE != 2>(s1, s1);
                const uint32_t s = kb % kStages;
                bool ok = true;
                if (kb >= kStages) {
                    if (lane == 0) ok = mbar_wait(&tail->empty[s], ((kb / kStages) - 1u) & 1u, err);
                    ok = __shfl_sync(0xffffffffu, ok, 0);
                }
                if (!ok) *abort_flag = 1;
                if (*abort_flag) {
                    stop6 = true;
                    break;
                }
                if (MODE == 2)
                    dequant_q6_quarter_x3(ql, shl, qh, shh, 4u * (sub & 1u), 2u * q, s0, s1, nrow, hi,
                                          smem + s * kStageBytes + kBOff, smem + s * kStageBytes + kBOff + kBTile);
                else
                    dequant_q6_quarter<F16>(ql, shl, qh, shh, 4u * (sub & 1u), 2u * q, f0, f1, nrow, hi,
                                            smem + s * kStageBytes + kBOff);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor-core reads
                __syncwarp();
                if (lane == 0) mbar_arrive(&tail->full_b[s]);
              }
            }
        } else {
            // the code bytes of stage kb are loaded kPrefetch stages ahead, so
            // global-memory latency overlaps the dequantisation of earlier stages;
            // scales are unpacked once per super-block (every 4 stages)
            constexpr uint32_t kPrefetch = 4;
            uint4 pq0[kPrefetch], pq1[kPrefetch];
            auto load_codes = [&](uint32_t kb, uint4& a, uint4& b) {
                const uint8_t* blk = row + (kb >> 2) * 144u + 16u + 32u * (kb & 3u);
                a = ld_nc_v4(blk);
                b = ld_nc_v4(blk + 16u);
            };
    #pragma unroll
            for (uint32_t i = 0; i < kPrefetch; ++i)
                if (i < nkb) load_codes(i, pq0[i], pq1[i]);
            uint4 hd_next = ld_nc_v4(row);
            uint32_t fb[4], ob[4];
            float ff[4], of[4];
            bool stop = false;
            for (uint32_t kb0 = 0; kb0 < nkb && !stop; kb0 += kPrefetch) {  // kPrefetch == 4: one super-block
                if (MODE == 2)
                    subblock_consts_f32(hd_next, hi, ff, of);
                else
                    subblock_consts<F16>(hd_next, hi, fb, ob);
                if (kb0 + 4u < nkb) hd_next = ld_nc_v4(row + ((kb0 >> 2) + 1u) * 144u);
    #pragma unroll
                for (uint32_t i = 0; i < kPrefetch; ++i) {
                    const uint32_t kb = kb0 + i;
                    if (kb >= nkb) break;
                    const uint4 c0 = pq0[i], c1 = pq1[i];
                    if (kb + kPrefetch < nkb) load_codes(kb + kPrefetch, pq0[i], pq1[i]);
                    const uint32_t s = kb % kStages;
                    bool ok = true;
                    if (kb >= kStages) {
                        if (lane == 0) ok = mbar_wait(&tail->empty[s], ((kb / kStages) - 1u) & 1u, err);
                        ok = __shfl_sync(0xffffffffu, ok, 0);
                    }
                    if (!ok) *abort_flag = 1;
                    if (*abort_flag) {
                        stop = true;
                        break;
                    }
                    if (MODE == 2)
                        dequant_subblock_x3(c0, c1, ff[i], of[i], nrow, hi, smem + s * kStageBytes + kBOff,
                                            smem + s * kStageBytes + kBOff + kBTile);
                    else
                        dequant_subblock<F16>(c0, c1, fb[i], ob[i], nrow, hi, smem + s * kStageBytes + kBOff);
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor-core reads
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tail->full_b[s]);
                }
            }
        }
        // epilogue: warp (2..5) % 4 owns TMEM lanes 32*q .. 32*q+31
        const bool ok = mbar_wait(&tail->done, 0, err);
        asm volatile("tcgen05.fence::after_thread_sync;");
        const uint32_t q = warp & 3u, sub = (warp - 2u) >> 2;  // lane quarter; which of its warps
        const bool store = ok && !*abort_flag;
        constexpr uint32_t kPairs = 2u * (kBN / 32u), kPerQuarter = kDqWarps / 4u;
        // accumulators -> y (single split) or -> this split's partial tile
        float* dst_base = sk.ks == 1u ? y : sk.ws + (uint64_t)split * m * n_total;
#pragma unroll 1
        for (uint32_t pair = sub; pair < kPairs; pair += kPerQuarter) {
            const uint32_t acc = pair / (kBN / 32u), cb = pair % (kBN / 32u);
            uint32_t r[32];
            tmem_ld32(tmem + ((32u * q) << 16) + acc * 128u + cb * 32u, r);
            const uint32_t mrow = acc * 128u + 32u * q + lane;
            if (store && mrow < m) {
                const uint64_t off = (uint64_t)mrow * n_total + n0 + cb * 32u;
                float4* dst = reinterpret_cast<float4*>(dst_base + off);
                const bool add_res = residual && sk.ks == 1u;  // y = residual + x W^T (split: after the sum)
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    float4 v = make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]),
                                           __uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3]));
                    if (add_res) {
                        const float4 rr = reinterpret_cast<const float4*>(residual + off)[i];
                        v = make_float4(rr.x + v.x, rr.y + v.y, rr.z + v.z, rr.w + v.w);
                    }
                    dst[i] = v;
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

// y = (residual +) sum over splits of ws[split] -- float4 by float4 over the
// whole m x n output, splits added in order.
__global__ void __launch_bounds__(256) gemm_splitk_reduce_kernel(const float4* __restrict__ ws, uint32_t ks,
                                                                 uint64_t n4, const float4* __restrict__ residual,
                                                                 float4* __restrict__ y) {
    pdl_wait();  // the partials come from the GEMM launch before
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (uint64_t)gridDim.x * blockDim.x) {
        float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
        for (uint32_t sp = 0; sp < ks; ++sp) {
            const float4 v = ws[(uint64_t)sp * n4 + i];
            t.x += v.x, t.y += v.y, t.z += v.z, t.w += v.w;
        }
        if (residual) {
            const float4 r = residual[i];
            t = make_float4(r.x + t.x, r.y + t.y, r.z + t.z, r.w + t.w);
        }
        y[i] = t;
    }
}

// The same reduce, the output rows of this rank's shard (columns [c0, c0 + n) of an
// m x n_total result) stored into EVERY rank's result -- local stores for its own,
// NVLink peer stores for the others, float4 by float4, nothing read from a peer --
// then the ranks' flag handshake (rank_flag_handshake) run by the warp of the CTA
// that completes the counter: when the launch ends on rank r, y[r] holds all
// n_total columns.  The fused form of GEMM + all-gather for output-row-sharded
// prefill projections.
struct GemmGather {
    float* y[8];           // rank q's m x n_total result, as this process maps it
    uint32_t* flags[8];    // rank q's flag array
    uint32_t* ctr;         // this rank's CTA counter (zero between launches)
    uint32_t n_ranks, rank, epoch, c0, n_total;
    unsigned long long wait_ns;
};

__global__ void __launch_bounds__(256) gemm_reduce_gather_kernel(const float4* __restrict__ ws, uint32_t ks,
                                                                 uint32_t n4_row, uint64_t n4,
                                                                 const GemmGather g, unsigned int* err) {
    pdl_wait();  // the partials come from the GEMM launch before
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (uint64_t)gridDim.x * blockDim.x) {
        float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
        for (uint32_t sp = 0; sp < ks; ++sp) {
            const float4 v = ws[(uint64_t)sp * n4 + i];
            t.x += v.x, t.y += v.y, t.z += v.z, t.w += v.w;
        }
        const uint64_t row = i / n4_row, c4 = i - row * n4_row;
        const uint64_t off = (row * g.n_total + g.c0) / 4u + c4;  // float4 index in every rank's result
#pragma unroll
        for (uint32_t q = 0; q < 8; ++q)
            if (q < g.n_ranks) reinterpret_cast<float4*>(g.y[q])[off] = t;
    }
    __threadfence_system();  // this thread's (peer) stores before the CTA's count
    __syncthreads();
    if (threadIdx.x < 32) {
        uint32_t last = 0;
        if (threadIdx.x == 0) last = atomicAdd(g.ctr, 1u) == gridDim.x - 1u ? 1u : 0u;
        if (__shfl_sync(0xffffffffu, last, 0)) {
            if (threadIdx.x == 0) *g.ctr = 0u;  // re-armed for the next launch in stream order
            rank_flag_handshake(g.flags, g.n_ranks, g.rank, g.epoch, g.wait_ns, err);
        }
    }
}

struct GemmScratch {
    float* ws = nullptr;
    size_t ws_floats = 0;
};
std::mutex g_gemm_mutex;
GemmScratch g_gemm_scratch[64];

// Per-device split-K scratch, grown on demand (not while a graph is being
// captured; split-K launches on one device must not overlap in time).
int gemm_splitk_reserve(size_t ws_floats, float** ws) {
    const int slot = device_slot();
    if (slot < 0) return set_error(ARC_E_CUDA, "gemm split-K scratch: no current device below index 64");
    std::lock_guard<std::mutex> lock(g_gemm_mutex);
    GemmScratch& g = g_gemm_scratch[slot];
    if (g.ws_floats < ws_floats) {
        float* nws = nullptr;
        cudaError_t e = cudaMalloc(&nws, ws_floats * sizeof(float));
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e != cudaSuccess) {
            cudaFree(nws);
            return set_cuda_error(e, "gemm split-K scratch");
        }
        cudaFree(g.ws);
        g.ws = nws;
        g.ws_floats = ws_floats;
    }
    *ws = g.ws;
    return ARC_OK;
}

}  // namespace

int gemm_q4k_bf16_prepare() {
    static std::atomic<bool> done[64] = {};
    static std::mutex prep_mutex;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return set_error(ARC_E_CUDA, "gemm prepare: no current device below index 64");
    if (done[dev].load(std::memory_order_acquire)) return ARC_OK;
    std::lock_guard<std::mutex> lock(prep_mutex);
    if (done[dev].load(std::memory_order_relaxed)) return ARC_OK;
    cudaError_t e = cudaSuccess;
    auto attr = [&](auto kern, uint32_t bytes) {
        if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    };
    attr(gemm_kq_bf16_kernel<12, 0>, smem_bytes<0>());
    attr(gemm_kq_bf16_kernel<14, 0>, smem_bytes<0>());
    attr(gemm_kq_bf16_kernel<12, 1>, smem_bytes<1>());
    attr(gemm_kq_bf16_kernel<14, 1>, smem_bytes<1>());
    attr(gemm_kq_bf16_kernel<12, 2>, smem_bytes<2>());
    attr(gemm_kq_bf16_kernel<14, 2>, smem_bytes<2>());
    if (e != cudaSuccess) return set_cuda_error(e, "gemm prepare");
    done[dev].store(true, std::memory_order_release);
    return ARC_OK;
}

namespace {
// Tensor map of an m x k row-major 16-bit activation, 64 x 128 boxes, 128-byte swizzle.
int encode_x_map(EncodeTiledFn enc, const uint16_t* x, uint32_t k, uint32_t m, bool fp16, CUtensorMap* map) {
    const cuuint64_t dims[2] = {k, m};
    const cuuint64_t strides[1] = {(cuuint64_t)k * 2u};
    const cuuint32_t box[2] = {kBK, 128};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(map, fp16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                           const_cast<uint16_t*>(x), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? ARC_OK : set_error(ARC_E_INVALID_ARGUMENT, "gemm: tensor map for X rejected");
}
}  // namespace

namespace {
int gemm_kq_impl(int fmt, const void* w, uint32_t n, uint32_t k, const uint16_t* x, uint32_t m,
                 const float* residual, float* y, cudaStream_t stream, int mode, const uint16_t* x_lo,
                 const GemmGather* gather) {
    if (fmt != 12 && fmt != 14) return set_error(ARC_E_INVALID_ARGUMENT, "gemm: weights must be Q4_K or Q6_K");
    if (mode < 0 || mode > 2) return set_error(ARC_E_INVALID_ARGUMENT, "gemm: operand mode 0 (bf16), 1 or 2 (fp16)");
    if (!w || !x || (!y && !gather) || (mode == 2 && !x_lo))
        return set_error(ARC_E_INVALID_ARGUMENT, "gemm: null pointer");
    if (m == 0 || m > 256 || n == 0 || n % kBN || k == 0 || k % 256u)
        return set_error(ARC_E_UNSUPPORTED_SHAPE, "gemm: needs 1 <= M <= 256, N % 128 == 0, K % 256 == 0");
    if ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) |
         reinterpret_cast<uintptr_t>(residual) | reinterpret_cast<uintptr_t>(x_lo)) & 15u)
        return set_error(ARC_E_ALIGNMENT, "gemm: W, X, residual and Y must be 16-byte aligned");
    int st = gemm_q4k_bf16_prepare();
    if (st != ARC_OK) return st;
    EncodeTiledFn enc = encode_tiled_fn();
    if (!enc) return set_error(ARC_E_CUDA, "gemm: cuTensorMapEncodeTiled unavailable");
    CUtensorMap map, map_lo;
    st = encode_x_map(enc, x, k, m, mode >= 1, &map);
    if (st == ARC_OK) st = encode_x_map(enc, mode == 2 ? x_lo : x, k, m, mode >= 1, &map_lo);
    if (st != ARC_OK) return st;
    // split K so that about one CTA per SM is busy (whole super-blocks per split)
    int dev = 0;
    cudaGetDevice(&dev);
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const uint32_t tiles = n / kBN;
    uint32_t ks = std::max(1u, std::min((uint32_t)sms / tiles, k / 256u));
    // tuning override for experiments: ARCLLM_GEMM_KS=<splits> (1 .. K/256)
    if (const char* ev = std::getenv("ARCLLM_GEMM_KS")) {
        const uint32_t f = (uint32_t)std::strtoul(ev, nullptr, 10);
        if (f >= 1u && f <= k / 256u) ks = f;
    }
    SplitKWs sk{nullptr, ks};
    if (ks > 1 || gather) {  // the gather form always reduces out of the scratch (one split: a copy)
        st = gemm_splitk_reserve((size_t)ks * m * n, &sk.ws);
        if (st != ARC_OK) return st;
        if (ks == 1) y = sk.ws;  // the single split's tile lands in the scratch
    }
    const uint8_t* wb = static_cast<const uint8_t*>(w);
    const dim3 grid(tiles, ks), block(kThreads);
    unsigned int* err = dev_error_word();
    cudaError_t e;
#define ARC_GEMM_LAUNCH(F, M)                                                                                   \
    launch_kernel(gemm_kq_bf16_kernel<F, M>, grid, block, smem_bytes<M>(), stream, map, map_lo, wb, n, k, m, \
                  residual, y, err, sk)
    if (fmt == 12)
        e = mode == 0 ? ARC_GEMM_LAUNCH(12, 0) : mode == 1 ? ARC_GEMM_LAUNCH(12, 1) : ARC_GEMM_LAUNCH(12, 2);
    else
        e = mode == 0 ? ARC_GEMM_LAUNCH(14, 0) : mode == 1 ? ARC_GEMM_LAUNCH(14, 1) : ARC_GEMM_LAUNCH(14, 2);
#undef ARC_GEMM_LAUNCH
    if (e == cudaSuccess && gather) {
        const uint64_t n4 = (uint64_t)m * n / 4u;
        const uint32_t blocks = (uint32_t)std::min<uint64_t>((n4 + 255) / 256, (uint64_t)sms * 8u);
        e = launch_kernel(gemm_reduce_gather_kernel, dim3(blocks), dim3(256), 0, stream,
                          reinterpret_cast<const float4*>(sk.ws), ks, n / 4u, n4, *gather, err);
    } else if (e == cudaSuccess && ks > 1) {
        const uint64_t n4 = (uint64_t)m * n / 4u;
        const uint32_t blocks = (uint32_t)std::min<uint64_t>((n4 + 255) / 256, (uint64_t)sms * 8u);
        e = launch_kernel(gemm_splitk_reduce_kernel, dim3(blocks), dim3(256), 0, stream,
                          reinterpret_cast<const float4*>(sk.ws), ks, n4, reinterpret_cast<const float4*>(residual),
                          reinterpret_cast<float4*>(y));
    }
    return e == cudaSuccess ? ARC_OK : set_cuda_error(e, "gemm launch");
}
}  // namespace

int gemm_kq_bf16(int fmt, const void* w, uint32_t n, uint32_t k, const uint16_t* x, uint32_t m,
                 const float* residual, float* y, cudaStream_t stream, int mode, const uint16_t* x_lo) {
    return gemm_kq_impl(fmt, w, n, k, x, m, residual, y, stream, mode, x_lo, nullptr);
}

// Exchange buffer of one rank for the gathered GEMM: the m x n_total fp32 result at 0, then at a
// 256-byte boundary the flag array (8 u32) and, 64 bytes further, the CTA counter.
uint64_t gemm_gather_flags_offset(uint32_t m, uint32_t n_total) {
    return ((uint64_t)m * n_total * 4u + 255u) & ~uint64_t(255);
}

int gemm_kq_allgather(int fmt, const void* w, uint32_t n, uint32_t k, const uint16_t* x, uint32_t m, uint32_t c0,
                      uint32_t n_total, void* const* rank_bufs, uint32_t n_ranks, uint32_t rank, uint32_t epoch,
                      uint32_t timeout_us, cudaStream_t stream) {
    if (!rank_bufs || n_ranks == 0 || n_ranks > 8 || rank >= n_ranks || epoch == 0 || (uint64_t)c0 + n > n_total ||
        c0 % 4u || n_total % 4u)
        return set_error(ARC_E_INVALID_ARGUMENT, "gemm all-gather: bad rank layout, columns or epoch");
    GemmGather g{};
    const uint64_t fo = gemm_gather_flags_offset(m, n_total);
    for (uint32_t q = 0; q < n_ranks; ++q) {
        if (!rank_bufs[q] || (reinterpret_cast<uintptr_t>(rank_bufs[q]) & 255u))
            return set_error(ARC_E_ALIGNMENT, "gemm all-gather: rank buffers must be 256-byte aligned");
        uint8_t* b = static_cast<uint8_t*>(rank_bufs[q]);
        g.y[q] = reinterpret_cast<float*>(b);
        g.flags[q] = reinterpret_cast<uint32_t*>(b + fo);
    }
    g.ctr = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(rank_bufs[rank]) + fo + 64u);
    g.n_ranks = n_ranks;
    g.rank = rank;
    g.epoch = epoch;
    g.c0 = c0;
    g.n_total = n_total;
    g.wait_ns = 1000ull * (timeout_us ? timeout_us : 2000000u);
    return gemm_kq_impl(fmt, w, n, k, x, m, nullptr, nullptr, stream, 0, nullptr, &g);
}

int gemm_q4k_bf16(const void* w, uint32_t n, uint32_t k, const uint16_t* x, uint32_t m, float* y,
                  cudaStream_t stream) {
    return gemm_kq_bf16(12, w, n, k, x, m, nullptr, y, stream);
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda
// symbol dependence at load time); null when the driver does not provide it.
EncodeTiledFn encode_tiled_fn() {
    static EncodeTiledFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

}  // namespace arc
