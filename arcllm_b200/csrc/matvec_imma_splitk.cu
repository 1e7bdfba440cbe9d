// Integer-MMA matvec for long rows (K > 3584: the FFN down projection
// 3584 x 18944), B200 (sm_100a).
//
// K is cut into P slices of at most 14 super-blocks (an even number for
// Q6_K).  Every CTA works on ONE slice for a contiguous range of row groups,
// so it runs the whole-row kernel's consumer scheme unchanged: consumer warp
// w owns super-block w of its slice (Q6_K: half 0 of block w and half 1 of
// block w^1) for the whole kernel and keeps its routed x fragments and scale
// constants in registers.  The host gives each slice a share of the SMs in
// proportion to its width and picks P so that the busiest CTA streams as few
// bytes as possible (3584 rows are 112 groups of 32: no split of whole rows
// balances them over 148 SMs, slices of rows do).
//
// Stages: G = 32 rows x one slice, loaded with 2-D tensor TMA boxes.  The
// matrix is viewed as u64 words in "super-rows" of Rs rows (Q4_K: Rs = 1;
// Q6_K: Rs = 4, because 15540-byte rows are 4 mod 16 bytes and only every
// fourth row starts on the 16-byte boundary a tensor-map stride needs).  One
// box takes one column of the slice (<= 2 KB of each row: <= 14 Q4_K or 8
// Q6_K blocks, from the 16-byte boundary below the column) for every Rs-th
// row of the group, so a Q4_K stage is ONE TMA operation and a Q6_K stage
// 4 x (1 or 2 columns).  Measured on B200, one 1-D bulk copy per row-slice
// (1-3 KB each) streamed at only ~110 ns per copy per SM (1.7-3.5 TB/s with
// the consumers switched off) and 16-byte cp.async from one warp was slower
// still: the copy engine wants few large operations.  Boxes land densely in
// shared memory ([i][j] rows of a column region); box widths are padded so
// that consecutive rows of one LDS sit 4 words (Q6_K, 32-bit reads of rows
// 4g+m) or 8 words (Q4_K, 64-bit reads) apart mod 32 banks.  Rows of a Q6_K
// matrix must come in multiples of 4; rows past the end of the matrix are
// zero-filled by the TMA unit and never stored.
//
// Reduction: the producer warp adds the consumer warps' row partials in warp
// order and stores the CTA's slice partial to a per-device scratch as 64-bit
// words tagged with the launch's tag (a device counter read after
// griddepcontrol.wait and advanced by the launch's last CTA out).  Row group g
// is closed by the CTA of slice g % P that owns it: its idle consumer warps
// read the P slice words of each row until all carry the tag, add them in
// slice order -- deterministic whichever slice came last -- apply bias /
// residual and write y.  Every word is its own flag: no fence and no arrival
// counter on the critical path (measured on B200, the fence + counter close
// it replaces cost Q6_K 3584 x 18944 18.2 against 16.9 us).
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "arcllm_cuda_internal.h"
#include "common.cuh"
#include "matvec_common.cuh"
#include "matvec_imma.cuh"

namespace arc {
namespace {

constexpr uint32_t kMaxSlices = 16;
constexpr uint32_t kMaxMaps = 4;
constexpr uint32_t kNW = 14;                         // consumer warps = widest slice
constexpr uint32_t kG = 32;                          // rows per stage (two 16-row MMA tiles)
constexpr uint32_t kXScratch = 1024;                 // per consumer warp: 3 limb planes + window constants
constexpr uint32_t kHead = 2 * kMaxStages * 8 + 16;  // full/empty barriers, abort flag, launch tag (+pad)
constexpr uint32_t kBoxMax = 2048;                   // bytes: 256 u64 elements per box row

struct KSlice {
    unsigned long long* part;  // [P][rows] slice partials, (tag << 32 | fp32 bits)
    uint32_t* ctl;             // [0] launch counter (tag = ctl[0] + 1), [1] CTAs counted out (zero between launches)
    uint32_t P, tx_max;
    uint16_t kb0[kMaxSlices], W[kMaxSlices], cta0[kMaxSlices + 1];
    // per slice: columns (1 or 2) = (first block in the slice, box bytes, map, smem region offset)
    uint8_t ncol[kMaxSlices], cst[kMaxSlices][2], cmap[kMaxSlices][2];
    uint16_t cbw[kMaxSlices][2];
    uint32_t coff[kMaxSlices][2], tx[kMaxSlices];
};

struct __align__(64) KMaps {
    CUtensorMap m[kMaxMaps];
};

// One CTA's slice, read out of the parameter tables with compile-time
// indices only (a runtime index into a kernel parameter array makes the
// compiler copy the array to local memory).
struct SliceView {
    uint32_t sl, W, kb0, C, ci, ncol, tx;
    uint32_t cst[2], cbw[2], coff[2], cmap[2];
};

__device__ __forceinline__ SliceView slice_of(const KSlice& q, uint32_t bid) {
    SliceView v{};
#pragma unroll
    for (uint32_t i = 0; i < kMaxSlices; ++i) {
        if (i < q.P && q.cta0[i] <= bid && bid < q.cta0[i + 1]) {
            v.sl = i;
            v.W = q.W[i];
            v.kb0 = q.kb0[i];
            v.C = q.cta0[i + 1] - q.cta0[i];
            v.ci = bid - q.cta0[i];
            v.ncol = q.ncol[i];
            v.tx = q.tx[i];
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                v.cst[c] = q.cst[i][c];
                v.cbw[c] = q.cbw[i][c];
                v.coff[c] = q.coff[i][c];
                v.cmap[c] = q.cmap[i][c];
            }
        }
    }
    return v;
}

__host__ __device__ constexpr uint32_t ks_red_off() { return kHead + 32 * 8; }
__host__ __device__ constexpr uint32_t ks_xscr_off(uint32_t S) {
    return (ks_red_off() + 2 * S * kNW * kG * 4 + 15u) & ~15u;
}
__host__ __device__ constexpr uint32_t ks_stage_off(uint32_t S) { return ks_xscr_off(S) + kNW * kXScratch; }

__device__ __forceinline__ void tma_box_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                           uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// Round `itr` of this CTA (row group grp) is complete: add the consumer
// warps' partials in warp order and store the CTA's slice partial of the
// group's rows as words tagged with this launch's tag.  Run by the producer.
__device__ __forceinline__ void ks_partial(const MvParams& p, const KSlice& q, const float* red, uint32_t W,
                                           uint32_t sl, uint32_t itr, uint32_t grp, uint32_t lane, uint32_t tag) {
    const uint32_t S = p.stages, s = itr % S, par = (itr / S) & 1u;
    const uint32_t rows_g = min(kG, p.rows - grp * kG);
    const float* rs = red + (par * S + s) * kNW * kG;
    if (lane < rows_g) {
        float a = 0.f;
        for (uint32_t w = 0; w < W; ++w) a += rs[w * kG + lane];
        st_relaxed_gpu_u64(q.part + (size_t)sl * p.rows + grp * kG + lane,
                           ((unsigned long long)tag << 32) | __float_as_uint(a));
    }
}

// Closing a row group: the CTA of slice (group % P) that owns the group,
// once its own rounds are consumed, has consumer warp w take its groups w,
// w + W, ... among those; for each row (one per lane) the warp reads the P
// slice partials until every word carries this launch's tag, adds them in
// slice order (deterministic: the same order whichever slice came last),
// applies bias / residual and writes y.  No fence and no counter: each word is
// its own flag, and the close work is spread over the slices and the warps.
// Gives up after kWaitLimitNs.
__device__ __forceinline__ void ks_close(const MvParams& p, const KSlice& q, uint32_t sl, uint32_t g0, uint32_t n,
                                         uint32_t warp, uint32_t W, uint32_t lane, uint32_t tag) {
    const unsigned long long t0 = globaltimer();
    uint32_t k = 0;  // index among this CTA's groups that it closes
    for (uint32_t gi = 0; gi < n; ++gi) {
        const uint32_t grp = g0 + gi;
        if (grp % q.P != sl) continue;
        if (k++ % W != warp) continue;
        const uint32_t rows_g = min(kG, p.rows - grp * kG);
        const uint32_t row = grp * kG + lane;
        if (lane >= rows_g) continue;
        unsigned long long v[kMaxSlices];
#pragma unroll
        for (uint32_t j = 0; j < kMaxSlices; ++j)  // every slice's word in flight before the first wait
            if (j < q.P) v[j] = ld_relaxed_gpu_u64(q.part + (size_t)j * p.rows + row);
        float t = 0.f;
#pragma unroll
        for (uint32_t j = 0; j < kMaxSlices; ++j) {
            if (j >= q.P) break;
            while ((uint32_t)(v[j] >> 32) != tag) {
                if (globaltimer() - t0 > kWaitLimitNs) {
                    raise_error(p.err, ARC_DEV_ERR_TIMEOUT);
                    return;
                }
                __nanosleep(32);
                v[j] = ld_relaxed_gpu_u64(q.part + (size_t)j * p.rows + row);
            }
            t += __uint_as_float((uint32_t)v[j]);
        }
        if (p.bias) t += p.bias[row];
        if (p.residual) t = p.residual[row] + t;
        p.y[row] = t;
    }
}

// Producer lane 0 at the very end of every CTA: count the CTA out; the last
// one advances the launch counter (the next launch's tag) and re-arms the count.
// Every CTA of this launch read the counter before it counted out.
__device__ __forceinline__ void ks_count_out(const KSlice& q) {
    if (atomicAdd(q.ctl + 1, 1u) == gridDim.x - 1u) {
        q.ctl[1] = 0u;
        atomicAdd(q.ctl, 1u);
    }
}

// Block bytes and tensor-map super-row height per format: Q4_K 144 B rows of
// 16-byte multiples (Rs 1), Q6_K 210 B (rows 4 mod 16: Rs 4), the EXEC148
// image 148 B (rows of 74 blocks are 8 mod 16: Rs 2).
__host__ __device__ constexpr uint32_t ks_bsz(int fmt) { return fmt == 12 ? 144u : fmt == 14 ? 210u : 148u; }
__host__ __device__ constexpr uint32_t ks_rs(int fmt) { return fmt == 12 ? 1u : fmt == 14 ? 4u : 2u; }

// Lane 0 of a producer warp: the TMA boxes of row group grp of this CTA's
// slice into stage stg, completing on bar.
template <int FMT>
__device__ __forceinline__ void ks_issue(const MvParams& p, const SliceView& sv, const KMaps& maps, uint8_t* stg,
                                         uint64_t* bar, uint32_t grp, uint64_t pol) {
    constexpr uint32_t bsz = ks_bsz(FMT);
    constexpr uint32_t Rs = ks_rs(FMT);  // rows per tensor-map super-row
    constexpr uint32_t J = kG / Rs;      // box rows
    mbar_arrive_expect_tx(bar, sv.tx);   // whole boxes, zero-filled rows included
#pragma unroll
    for (uint32_t c = 0; c < 2; ++c) {
        if (c < sv.ncol) {
            const uint32_t mi = sv.cmap[c];
            const CUtensorMap* mp = mi == 0 ? &maps.m[0] : mi == 1 ? &maps.m[1] : mi == 2 ? &maps.m[2] : &maps.m[3];
            const uint32_t bw = sv.cbw[c];
#pragma unroll
            for (uint32_t i = 0; i < Rs; ++i) {
                const uint32_t xb = (uint32_t)(((uint64_t)i * p.rb + (uint64_t)(p.kb_base + sv.kb0 + sv.cst[c]) * bsz) &
                                               ~(uint64_t)15);
                tma_box_2d(stg + sv.coff[c] + i * J * bw, mp, (int)(xb / 8u), (int)(grp * J), bar, pol);
            }
        }
    }
}

// Consumer warp `warp` (< the slice width) of a K-slice CTA: builds its routed
// x fragments (x indexed by the full K, times `inv` and gamma when the RMSNorm
// is fused), then consumes rounds [it0, it0 + n) of the stage ring -- this
// CTA's row groups of its slice -- leaving per-row partials in `red` and
// releasing each stage.  LDCG: read x through L2 (x written by other CTAs of
// the same launch).
template <int FMT, bool LDCG>
__device__ __forceinline__ void ks_consume(const MvParams& p, const SliceView& sv, const uint8_t* stages,
                                           uint64_t* full, uint64_t* empty, volatile int* abort_flag, float* red,
                                           uint8_t* xscr, float inv, uint32_t it0, uint32_t n, uint32_t warp,
                                           uint32_t lane) {
    constexpr uint32_t bsz = ks_bsz(FMT);
    constexpr uint32_t Rs = ks_rs(FMT);
    constexpr uint32_t J = kG / Rs;
    const uint32_t S = p.stages, kb0 = sv.kb0;
    const uint32_t jw = lane >> 2, qd = lane & 3u;
    // this warp's super-block(s) of the slice: x slice, quantised, routed fragments
    const uint32_t bA = p.kb_base + kb0 + warp, bB = FMT == 14 ? p.kb_base + kb0 + (warp ^ 1u) : bA;
    XFrag f;
    {
        const uint32_t e0 = 256u * (jw < 4 ? bA : bB) + 32u * jw + 8u * qd;
        const float4 a0 = LDCG ? __ldcg(reinterpret_cast<const float4*>(p.x + e0))
                               : *reinterpret_cast<const float4*>(p.x + e0);
        const float4 a1 = LDCG ? __ldcg(reinterpret_cast<const float4*>(p.x + e0 + 4))
                               : *reinterpret_cast<const float4*>(p.x + e0 + 4);
        float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        if (p.gamma) {
            const float4 g0v = *reinterpret_cast<const float4*>(p.gamma + e0);
            const float4 g1v = *reinterpret_cast<const float4*>(p.gamma + e0 + 4);
            const float gv[8] = {g0v.x, g0v.y, g0v.z, g0v.w, g1v.x, g1v.y, g1v.z, g1v.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = (v[i] * inv) * gv[i];
        }
        uint8_t* xs = xscr + warp * kXScratch;
        float* kc = reinterpret_cast<float*>(xs + 768);
        quantize8<FMT>(v, lane, xs, kc);
        __syncwarp();
        if (FMT == ARC_TYPE_EXEC148)
            gather_xfrag_e148(xs, kc, lane, f);
        else
            gather_xfrag<FMT>(xs, kc, xs, kc, lane, f);
    }
    // this warp's column of the slice (Q6_K columns split at even blocks, so
    // blocks w and w^1 share one), and where a row of it sits in a stage:
    // region + (i * J + j) * bw + skew for row r = i + Rs * j
    const bool c1 = sv.ncol == 2 && warp >= sv.cst[1];
    const uint32_t cs = c1 ? sv.cst[1] : sv.cst[0];
    const uint32_t bw = c1 ? sv.cbw[1] : sv.cbw[0];
    const uint32_t coff = c1 ? sv.coff[1] : sv.coff[0];
    const uint32_t g = lane >> 2, t = lane & 3u;
    uint32_t rowA[2], rowB[2];  // stage offsets of tile m's rows (lanes g, lanes g+8); the same every round
#pragma unroll
    for (int m = 0; m < 2; ++m) {
        const uint2 rr = tile_rows<FMT, 2>(m, g);
        const uint32_t r2[2] = {rr.x, rr.y};
        uint32_t o[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t r = r2[h], i = r % Rs;
            const uint32_t mis = (uint32_t)(((uint64_t)i * p.rb + (uint64_t)(p.kb_base + kb0 + cs) * bsz) & 15u);
            o[h] = coff + (i * J + r / Rs) * bw + mis;
        }
        rowA[m] = o[0];
        rowB[m] = o[1];
    }
    const uint32_t offA = (warp - cs) * bsz, offB = (FMT == 14 ? ((warp ^ 1u) - cs) : (warp - cs)) * bsz;
    const bool oddA = FMT == 14 && (warp & 1u) != 0u;

    for (uint32_t it = it0; it < it0 + n; ++it) {
        const uint32_t s = it % S;
        if (!mbar_wait(&full[s], (it / S) & 1u, p.err)) *abort_flag = 1;
        if (*abort_flag) break;
        const uint8_t* st = stages + s * p.stage_smem;
        float y[2][2];
#pragma unroll
        for (int m = 0; m < 2; ++m) {
            y[m][0] = y[m][1] = 0.f;
            const uint32_t row0 = rowA[m], row1 = rowB[m];
            if (FMT == 12)
                q4_tile(st, row0 + offA, row1 + offA, t, f, y[m][0], y[m][1]);
            else if (FMT == ARC_TYPE_EXEC148)
                e148_tile(st, row0 + offA, row1 + offA, t, f, y[m][0], y[m][1]);
            else if (oddA)
                q6_tile_lowreg<true>(st, row0, row1, offA, offB, t, f, y[m][0], y[m][1]);
            else
                q6_tile_lowreg<false>(st, row0, row1, offA, offB, t, f, y[m][0], y[m][1]);
        }
        // sum the quad's four lanes; lanes t == 0 then hold this warp's partial of their rows
        float* rs = red + ((((it / S) & 1u) * S + s) * kNW + warp) * kG;
#pragma unroll
        for (int m = 0; m < 2; ++m) {
            const uint2 rr = tile_rows<FMT, 2>(m, g);
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                float v = y[m][r];
                v += __shfl_xor_sync(0xffffffffu, v, 1);
                v += __shfl_xor_sync(0xffffffffu, v, 2);
                if (t == 0) rs[r ? rr.y : rr.x] = v;
            }
        }
        __syncwarp();
        if (lane == 0) {
            __threadfence_block();
            mbar_arrive(&empty[s]);  // releases the stage and publishes this warp's partials
        }
    }
}

template <int FMT>
__global__ void __launch_bounds__((kNW + 1) * 32, 1)
    matvec_imma_kslice_kernel(const MvParams p, const __grid_constant__ KSlice q, const __grid_constant__ KMaps maps) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kMaxStages;
    volatile int* abort_flag = reinterpret_cast<int*>(empty + kMaxStages);
    double* red_d = reinterpret_cast<double*>(smem + kHead);     // [32]
    float* red = reinterpret_cast<float*>(smem + ks_red_off());  // [2][S][kNW][kG]
    uint8_t* xscr = smem + ks_xscr_off(p.stages);
    uint8_t* stages = smem_align_up<128>(smem, ks_stage_off(p.stages));
    // this launch's tag (the header word after the abort flag), stored by consumer warp 0 after
    // griddepcontrol.wait
    volatile uint32_t* tagp = reinterpret_cast<volatile uint32_t*>(empty + kMaxStages) + 1;

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    const uint32_t S = p.stages;
    // this CTA's slice and its contiguous range of row groups
    const SliceView sv = slice_of(q, blockIdx.x);
    const uint32_t sl = sv.sl, W = sv.W;
    const uint32_t g0 = (uint32_t)((uint64_t)p.n_groups * sv.ci / sv.C);
    const uint32_t n = (uint32_t)((uint64_t)p.n_groups * (sv.ci + 1) / sv.C) - g0;
    pdl_trigger();

    if (tid == kNW * 32) {
        for (uint32_t s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], W);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kNW) {
        // ---------------- producer ----------------
        const uint64_t pol = l2_evict_first_policy();
        if (!p.early) pdl_wait();
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
        for (; it < n; ++it) {
            const uint32_t s = it % S;
            if (it >= S && !released(it - S)) {
                ok = false;
                break;
            }
            if (lane == 0) ks_issue<FMT>(p, sv, maps, stages + s * p.stage_smem, &full[s], g0 + it, pol);
            __syncwarp();
            // (a released round implies consumer warp 0 has stored the tag)
            if (it >= S) ks_partial(p, q, red, W, sl, it - S, g0 + it - S, lane, *tagp);
        }
        if (ok) {
            for (uint32_t j = it > S ? it - S : 0; j < it; ++j) {
                if (!released(j)) {
                    ok = false;
                    break;
                }
                ks_partial(p, q, red, W, sl, j, g0 + j, lane, *tagp);
            }
        }
        if (!ok && lane == 0) {  // no box may still be landing in this CTA's smem at exit
            const uint32_t first = it > S ? it - S : 0;
            for (uint32_t j = first; j < it; ++j) mbar_wait(&full[j % S], (j / S) & 1u, p.err);
        }
        if (lane == 0) ks_count_out(q);
        return;
    }

    // ---------------- consumers ----------------
    pdl_wait();  // x, gamma, bias and residual come from the preceding kernels
    if (tid == 0) *tagp = *reinterpret_cast<volatile uint32_t*>(q.ctl) + 1u;  // before warp 0's first release
    float inv = 1.0f;
    if (p.gamma) {  // fused RMSNorm over all of K (every consumer warp takes part)
        const uint32_t jw = lane >> 2, qd = lane & 3u;
        double ss = 0.0;
        for (uint32_t sb = warp; sb < p.nb; sb += kNW) {
            const uint32_t e0 = 256u * sb + 32u * jw + 8u * qd;
            const float4 a0 = *reinterpret_cast<const float4*>(p.x + e0);
            const float4 a1 = *reinterpret_cast<const float4*>(p.x + e0 + 4);
            ss += (double)a0.x * a0.x + (double)a0.y * a0.y + (double)a0.z * a0.z + (double)a0.w * a0.w;
            ss += (double)a1.x * a1.x + (double)a1.y * a1.y + (double)a1.z * a1.z + (double)a1.w * a1.w;
        }
        ss = warp_sum_d(ss);
        if (lane == 0) red_d[warp] = ss;
        named_bar_sync(1, kNW * 32u);
        double tot = 0.0;
        for (uint32_t w = 0; w < kNW; ++w) tot += red_d[w];
        inv = 1.0f / sqrtf((float)(tot / (double)p.k) + p.eps);
    }
    if (warp >= W) return;  // narrower slice: this warp has no super-block
    ks_consume<FMT, false>(p, sv, stages, full, empty, abort_flag, red, xscr, inv, 0u, n, warp, lane);
    if (!*abort_flag) ks_close(p, q, sl, g0, n, warp, W, lane, *tagp);
}

struct KsScratch {
    unsigned long long* part = nullptr;  // tagged slice partials
    uint32_t* ctl = nullptr;             // launch counter + CTA count-out
    size_t part_words = 0;
};
std::mutex g_ks_mutex;
KsScratch g_ks[64];

struct KsPlan {
    uint32_t S = 0, stage_smem = 0, smem = 0, grid = 0, n_groups = 0, nmaps = 0;
    uint32_t map_bw[kMaxMaps] = {};  // box bytes of each tensor map
    KSlice q{};
    bool ok = false;
};

// Box bytes for a column of `wb` blocks: room for the widest 16-byte skew,
// then padded so that consecutive rows of one LDS fall into distinct banks
// (Q4_K: 8 or 24 words mod 32 for the 64-bit half-warp reads; Q6_K: an odd
// multiple of 4 words for rows 4 apart).
uint32_t ks_box_bytes(int fmt, uint32_t wb) {
    const uint32_t bsz = ks_bsz(fmt);
    uint32_t bw = (wb * bsz + (fmt == 12 ? 0u : 12u) + 15u) & ~15u;
    if (fmt != 14)
        while ((bw / 4u) % 32u != 8u && (bw / 4u) % 32u != 24u) bw += 16u;
    else
        while (((bw / 16u) & 1u) == 0u) bw += 16u;
    return bw;
}

// Slices and CTA shares for one shape: for each candidate slice count P the
// widths are as even as possible (pairs of blocks for Q6_K), CTAs go one at a
// time to the slice whose busiest CTA has the most work, and the P with the
// least work on the busiest CTA wins.  Work = row groups x (width + 6): a row
// segment costs about as much as six more blocks of it (measured on B200 with
// the FFN-down shape: 6 slices of 12-13 blocks beat 10 slices of 7-8 by 15 %).
// Each slice is then cut into at most two box columns of <= 2 KB per row.
KsPlan ks_plan(int fmt, uint32_t rows, uint32_t k, uint32_t sms) {
    KsPlan pl{};
    const uint32_t nb = k / 256u, unit = fmt == 14 ? 2u : 1u, nu = nb / unit, wmax_u = kNW / unit;
    pl.n_groups = (rows + kG - 1u) / kG;
    uint64_t best = ~0ull;
    uint32_t p_lo = (nu + wmax_u - 1u) / wmax_u;
    uint32_t p_hi = std::min<uint32_t>(std::min<uint32_t>(kMaxSlices, nu), std::min<uint32_t>(p_lo + 4u, sms));
    // tuning override for experiments: ARCLLM_KSLICE_P=<slice count> (kept within the legal range)
    if (const char* e = std::getenv("ARCLLM_KSLICE_P")) {
        const uint32_t f = (uint32_t)std::strtoul(e, nullptr, 10);
        if (f >= p_lo && f <= std::min<uint32_t>(kMaxSlices, nu)) p_lo = p_hi = f;
    }
    for (uint32_t P = p_lo; P <= p_hi; ++P) {
        uint32_t W[kMaxSlices], C[kMaxSlices];
        for (uint32_t i = 0; i < P; ++i) {
            W[i] = (nu / P + (i < nu % P ? 1u : 0u)) * unit;
            C[i] = 1u;
        }
        auto cost = [&](uint32_t i) { return (uint64_t)(W[i] + 6u) * ((pl.n_groups + C[i] - 1u) / C[i]); };
        for (uint32_t total = P; total < sms; ++total) {
            uint32_t bi = P;
            for (uint32_t i = 0; i < P; ++i)
                if (C[i] < pl.n_groups && (bi == P || cost(i) > cost(bi))) bi = i;
            if (bi == P) break;
            ++C[bi];
        }
        uint64_t mx = 0;
        for (uint32_t i = 0; i < P; ++i) mx = std::max(mx, cost(i));
        if (mx < best) {
            best = mx;
            pl.q.P = P;
            uint32_t kb = 0, c0 = 0;
            for (uint32_t i = 0; i < P; ++i) {
                pl.q.kb0[i] = (uint16_t)kb;
                pl.q.W[i] = (uint16_t)W[i];
                pl.q.cta0[i] = (uint16_t)c0;
                kb += W[i];
                c0 += C[i];
            }
            pl.q.cta0[P] = (uint16_t)c0;
            pl.grid = c0;
        }
    }
    // box columns: Q4_K one (14 x 144 B = 2016 B fits a box row), Q6_K up to
    // two of <= 8 blocks, split in pairs as evenly as possible
    const uint32_t colmax = fmt == 12 ? kNW : fmt == 14 ? 8u : 13u;  // box rows of <= 2 KB
    uint32_t stage = 0;
    for (uint32_t s = 0; s < pl.q.P; ++s) {
        const uint32_t Wd = pl.q.W[s];
        const uint32_t ncol = (Wd + colmax - 1u) / colmax;
        uint32_t wcol[2] = {Wd, 0u};
        if (ncol == 2) {
            if (fmt == 14) {
                const uint32_t pairs = Wd / 2u;
                wcol[0] = 2u * ((pairs + 1u) / 2u);
            } else {
                wcol[0] = (Wd + 1u) / 2u;
            }
            wcol[1] = Wd - wcol[0];
        }
        pl.q.ncol[s] = (uint8_t)ncol;
        uint32_t off = 0, cst = 0;
        for (uint32_t c = 0; c < ncol; ++c) {
            const uint32_t bw = ks_box_bytes(fmt, wcol[c]);
            if (bw > kBoxMax) return pl;
            uint32_t mi = 0;
            while (mi < pl.nmaps && pl.map_bw[mi] != bw) ++mi;
            if (mi == pl.nmaps) {
                if (pl.nmaps == kMaxMaps) return pl;
                pl.map_bw[pl.nmaps++] = bw;
            }
            pl.q.cst[s][c] = (uint8_t)cst;
            pl.q.cmap[s][c] = (uint8_t)mi;
            pl.q.cbw[s][c] = (uint16_t)bw;
            pl.q.coff[s][c] = off;
            off += kG * bw;  // Rs boxes of kG / Rs rows
            cst += wcol[c];
        }
        pl.q.tx[s] = off;
        stage = std::max(stage, off);
    }
    pl.q.tx_max = stage;
    pl.stage_smem = (stage + 127u) & ~127u;
    uint32_t S = kMaxStages;
    while (S > 2 && ks_stage_off(S) + 128u + S * pl.stage_smem > 227u * 1024u) --S;
    pl.S = S;
    pl.smem = ks_stage_off(S) + 128u + S * pl.stage_smem;
    pl.ok = pl.smem <= 227u * 1024u;
    return pl;
}

// Plans are pure functions of the shape and SM count: cache them.
KsPlan ks_plan_cached(int fmt, uint32_t rows, uint32_t k, uint32_t sms) {
    struct Entry {
        int fmt;
        uint32_t rows, k, sms;
        KsPlan pl;
    };
    static std::mutex mu;
    static std::vector<Entry> cache;
    if (std::getenv("ARCLLM_KSLICE_P")) return ks_plan(fmt, rows, k, sms);  // tuning runs bypass the cache
    std::lock_guard<std::mutex> lock(mu);
    for (const Entry& e : cache)
        if (e.fmt == fmt && e.rows == rows && e.k == k && e.sms == sms) return e.pl;
    KsPlan pl = ks_plan(fmt, rows, k, sms);
    if (cache.size() >= 64) cache.erase(cache.begin());
    cache.push_back(Entry{fmt, rows, k, sms, pl});
    return pl;
}

int ks_sm_count() {
    static std::atomic<int> sm_count[64] = {};  // per device, queried once
    const int slot = device_slot();
    int sms = slot >= 0 ? sm_count[slot].load(std::memory_order_relaxed) : 0;
    if (sms > 0) return sms;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
        sms = 148;
    if (slot >= 0) sm_count[slot].store(sms, std::memory_order_relaxed);
    return sms;
}

template <int FMT>
cudaError_t set_attr_ks() {
    return cudaFuncSetAttribute(matvec_imma_kslice_kernel<FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                227 * 1024);
}

// The rows x k matrix as u64 words in super-rows of Rs rows (Rs * row bytes is a multiple of 16),
// one tensor map per box width of the plan.
int ks_encode_maps(int fmt, const void* w, uint32_t rows, uint32_t k, const KsPlan& pl, KMaps* maps) {
    EncodeTiledFn enc = encode_tiled_fn();
    if (!enc) return set_error(ARC_E_CUDA, "matvec split-K: cuTensorMapEncodeTiled unavailable");
    const uint32_t nb = k / 256u, rb = nb * ks_bsz(fmt), Rs = ks_rs(fmt);
    std::memset(maps, 0, sizeof *maps);
    for (uint32_t i = 0; i < pl.nmaps; ++i) {
        const cuuint64_t dims[2] = {(cuuint64_t)Rs * rb / 8u, (cuuint64_t)(rows / Rs)};
        const cuuint64_t strides[1] = {(cuuint64_t)Rs * rb};
        const cuuint32_t box[2] = {pl.map_bw[i] / 8u, kG / Rs};
        const cuuint32_t estr[2] = {1, 1};
        const CUresult r = enc(&maps->m[i], CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(w), dims, strides,
                               box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return set_error(ARC_E_INVALID_ARGUMENT, "matvec split-K: tensor map rejected");
    }
    return ARC_OK;
}

}  // namespace

int ks_reserve(int fmt, uint32_t rows, uint32_t k);

int matvec_splitk_reserve(int fmt, uint32_t rows, uint32_t k) {
    if (!matvec_splitk_supported(fmt, false, rows, k)) return ARC_OK;  // another kernel serves this shape
    return ks_reserve(fmt, rows, k);
}

int matvec_kwindow_reserve(int fmt, uint32_t rows, uint32_t nb_win) { return ks_reserve(fmt, rows, 256u * nb_win); }

// Scratch for the plan of (fmt, rows, k); k is the covered K (a window's width).
int ks_reserve(int fmt, uint32_t rows, uint32_t k) {
    const KsPlan pl = ks_plan_cached(fmt, rows, k, (uint32_t)ks_sm_count());
    if (!pl.ok) return set_error(ARC_E_UNSUPPORTED_SHAPE, "matvec split-K: no plan fits shared memory");
    const size_t need_part = (size_t)pl.q.P * rows;
    const int slot = device_slot();
    if (slot < 0) return set_error(ARC_E_CUDA, "matvec split-K: no current device below index 64");
    std::lock_guard<std::mutex> lock(g_ks_mutex);
    KsScratch& sc = g_ks[slot];
    if (sc.part_words >= need_part && sc.ctl) return ARC_OK;
    const size_t np = std::max(need_part, sc.part_words);
    unsigned long long* part = nullptr;
    uint32_t* ctl = nullptr;
    cudaError_t e = cudaMalloc(&part, np * sizeof(unsigned long long));
    if (e == cudaSuccess) e = cudaMalloc(&ctl, 4 * sizeof(uint32_t));
    // zeroed words carry tag 0, which no launch uses (tags start at 1)
    if (e == cudaSuccess) e = cudaMemset(part, 0, np * sizeof(unsigned long long));
    if (e == cudaSuccess) e = cudaMemset(ctl, 0, 4 * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaFree(part);
        cudaFree(ctl);
        return set_cuda_error(e, "matvec split-K scratch");
    }
    if (sc.ctl) {  // keep the launch counter running: words of earlier launches carry earlier tags
        e = cudaMemcpy(ctl, sc.ctl, sizeof(uint32_t), cudaMemcpyDeviceToDevice);
        if (e != cudaSuccess) {
            cudaFree(part);
            cudaFree(ctl);
            return set_cuda_error(e, "matvec split-K scratch");
        }
    }
    cudaFree(sc.part);  // grown only outside concurrent use (documented)
    cudaFree(sc.ctl);
    sc.part = part;
    sc.ctl = ctl;
    sc.part_words = np;
    return ARC_OK;
}

int matvec_splitk_prepare() {
    static std::atomic<bool> done[64] = {};  // concurrent first calls set the same (idempotent) attributes
    const int slot = device_slot();
    if (slot < 0) return set_error(ARC_E_CUDA, "matvec split-K prepare: no current device below index 64");
    if (done[slot].load(std::memory_order_acquire)) return ARC_OK;
    cudaError_t e = set_attr_ks<12>();
    if (e == cudaSuccess) e = set_attr_ks<14>();
    if (e == cudaSuccess) e = set_attr_ks<ARC_TYPE_EXEC148>();
    if (e != cudaSuccess) return set_cuda_error(e, "matvec split-K prepare");
    done[slot].store(true, std::memory_order_release);
    return ARC_OK;
}

// Single matrix, K > 3584; Q6_K: an even number of super-blocks and a
// multiple of 4 rows (the tensor-map super-rows).  The EXEC148 image (no
// whole-row form): any K, an even number of rows.
bool matvec_splitk_supported(int fmt, bool dual, uint32_t rows, uint32_t k) {
    if ((fmt != 12 && fmt != 14 && fmt != ARC_TYPE_EXEC148) || dual || rows == 0 || k % 256u) return false;
    const uint32_t nb = k / 256u;
    if (fmt == ARC_TYPE_EXEC148 && (rows & 1u)) return false;
    if ((fmt != ARC_TYPE_EXEC148 && nb <= 14) || (fmt == 14 && ((nb & 1u) || (rows & 3u)))) return false;
    if (nb > kNW * kMaxSlices) return false;
    return ks_plan_cached(fmt, rows, k, 148).ok;
}

int matvec_splitk_launch(int fmt, const void* w, uint32_t rows, uint32_t k, const float* x, const float* gamma,
                         float eps, const float* bias, const float* residual, float* y, cudaStream_t stream) {
    if (!matvec_splitk_supported(fmt, false, rows, k))
        return set_error(ARC_E_UNSUPPORTED_SHAPE, "matvec split-K: shape not supported");
    return matvec_kwindow_launch(fmt, w, rows, k, 0, k / 256u, x, gamma, eps, bias, residual, y, stream);
}

// Super-blocks [kb_base, kb_base + nb_win) of every row of a rows x k matrix:
// y[r] = residual[r] + bias[r] + sum over the window of W[r][.] * x[.] (x indexed
// by the full K).  The tensor-parallel decode runs the FFN down projection of
// its own slice of s this way.  Q6_K: kb_base and nb_win even, rows % 4 == 0;
// EXEC148: even rows.  No fused RMSNorm with a window.
int matvec_kwindow_launch(int fmt, const void* w, uint32_t rows, uint32_t k, uint32_t kb_base, uint32_t nb_win,
                          const float* x, const float* gamma, float eps, const float* bias, const float* residual,
                          float* y, cudaStream_t stream) {
    if ((fmt != 12 && fmt != 14 && fmt != ARC_TYPE_EXEC148) || rows == 0 || k % 256u || nb_win == 0 ||
        kb_base + nb_win > k / 256u || nb_win > kNW * kMaxSlices || (gamma && nb_win != k / 256u) ||
        (fmt == 14 && ((kb_base | nb_win) & 1u || (rows & 3u))) || (fmt == ARC_TYPE_EXEC148 && (rows & 1u)))
        return set_error(ARC_E_UNSUPPORTED_SHAPE, "matvec K window: shape not supported");
    const uint32_t kw = 256u * nb_win;
    if (!w || !x || !y) return set_error(ARC_E_INVALID_ARGUMENT, "matvec: null pointer");
    if (reinterpret_cast<uintptr_t>(w) & 15u)
        return set_error(ARC_E_ALIGNMENT, "matvec: weight pointers must be 16-byte aligned");
    int st = matvec_splitk_prepare();
    if (st == ARC_OK) st = ks_reserve(fmt, rows, kw);
    if (st != ARC_OK) return st;
    KsPlan pl = ks_plan_cached(fmt, rows, kw, (uint32_t)ks_sm_count());
    if (!pl.ok) return set_error(ARC_E_UNSUPPORTED_SHAPE, "matvec split-K: no plan fits shared memory");
    const uint32_t rb = (k / 256u) * ks_bsz(fmt);
    KMaps maps;
    st = ks_encode_maps(fmt, w, rows, k, pl, &maps);
    if (st != ARC_OK) return st;
    const int slot = device_slot();
    if (slot < 0) return set_error(ARC_E_CUDA, "matvec split-K: no current device below index 64");
    {
        std::lock_guard<std::mutex> lock(g_ks_mutex);
        pl.q.part = g_ks[slot].part;
        pl.q.ctl = g_ks[slot].ctl;
    }
    MvParams p{};
    p.w0 = static_cast<const uint8_t*>(w);
    p.x = x;
    p.gamma = gamma;
    p.eps = eps;
    p.bias = bias;
    p.residual = residual;
    p.y = y;
    p.err = dev_error_word();
    p.rows = rows;
    p.k = kw;
    p.nb = nb_win;
    p.rb = rb;
    p.kb_base = kb_base;
    p.G = kG;
    p.n_groups = pl.n_groups;
    p.stages = pl.S;
    p.stage_smem = pl.stage_smem;
    p.early = pdl_enabled() ? 1u : 0u;
    const dim3 block((kNW + 1) * 32);
    const cudaError_t e =
        fmt == 12   ? launch_kernel(matvec_imma_kslice_kernel<12>, dim3(pl.grid), block, pl.smem, stream, p, pl.q, maps)
        : fmt == 14 ? launch_kernel(matvec_imma_kslice_kernel<14>, dim3(pl.grid), block, pl.smem, stream, p, pl.q, maps)
                    : launch_kernel(matvec_imma_kslice_kernel<ARC_TYPE_EXEC148>, dim3(pl.grid), block, pl.smem, stream,
                                    p, pl.q, maps);
    return e == cudaSuccess ? ARC_OK : set_cuda_error(e, "matvec split-K launch");
}

}  // namespace arc
