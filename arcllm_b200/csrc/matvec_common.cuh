// Pieces shared by the streaming matvec kernels (matvec.cu: CUDA-core
// decode; matvec_mma.cu: tensor-core multiply-accumulate): the launch
// parameters, the TMA producer that streams row groups into the shared-memory
// ring, and the per-row butterfly fold.
#pragma once
#include <cstdint>

#include "common.cuh"

namespace arc {
namespace {

constexpr int kMaxStages = 8;
constexpr uint32_t kStagePad = 16;  // slack after each stage for 32-bit reads that run past a block

constexpr uint32_t kMaxRanks = 8;  // ranks of the all-gather epilogue (one node)

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
    uint32_t G;  // rows per group (<= template G)
    uint32_t n_groups;
    uint32_t stages;
    uint32_t stage_smem;  // bytes of one stage in smem (both matrices + pad)
    uint32_t x_floats;    // padded x length in smem
    uint32_t early;       // 1: weights may be streamed before the PDL wait (they are not written upstream)
    // fused RoPE / KV-store epilogue (whole-row integer-MMA kernel only; rope_mode 0 = none):
    // 1 rotate adjacent row pairs (2p, 2p+1) of each head_dim-row head at position *pos -> y;
    // 2 rotate, then store fp16 into cache row *pos; 3 store fp16 into cache row *pos
    uint32_t rope_mode, rope_half;  // rope_half = head_dim / 2
    const float2* rope_table;       // [max_ctx][head_dim/2] (cos, sin)
    const uint32_t* rope_pos;       // device position
    uint16_t* cache;                // cache base + layer offset; row `pos` starts at pos * rows
    uint32_t max_ctx;
    // rank all-gather epilogue (whole-row integer-MMA kernel, not dual, rope_mode 0; n_ranks 0 =
    // none), fence-free: row i of this shard goes to every rank q as ONE 64-bit word
    // (epoch << 32 | fp32 bits) at gather_ll[q][gather_row0 + i] (NVLink peer stores for q !=
    // self_rank); then every CTA reads its slice of this rank's word array until each word carries
    // `epoch` (at most wait_ns) and writes the values to gather_out[0, gather_rows_total)
    uint32_t n_ranks, self_rank, epoch;
    unsigned long long wait_ns;
    unsigned long long* gather_ll[kMaxRanks];
    const unsigned long long* gather_own;  // gather_ll[self_rank]
    float* gather_out;
    uint32_t gather_row0, gather_rows_total;
    // K-slice kernel only: the first super-block of the K window this launch covers
    // (the matrix rows keep their full length rb; nb counts the window's blocks)
    uint32_t kb_base;
    // several jobs in one launch (matvec_imma_multi_kernel): this job's CTAs are
    // [cta0, cta0 + ncta) of the grid; ncta 0 = the whole grid
    uint32_t cta0, ncta;
};

// This CTA's index within its job and the job's CTA count.
__device__ __forceinline__ uint32_t job_cta(const MvParams& p) { return p.ncta ? blockIdx.x - p.cta0 : blockIdx.x; }
__device__ __forceinline__ uint32_t job_ctas(const MvParams& p) { return p.ncta ? p.ncta : gridDim.x; }

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

template <int N>
constexpr int ilog2() {
    return N <= 1 ? 0 : 1 + ilog2<N / 2>();
}

// The producer warp: stream each row group assigned to this CTA into the
// stage ring with 1-D TMA bulk copies (one elected thread), waiting for the
// consumers to release a stage before refilling it.  Groups whose byte count
// is not a multiple of 16 (the ragged final Q6_K group) copy their tail by
// hand before arming the barrier.  On any timeout it sets *abort_flag, stops,
// and waits (bounded) for the copies it already issued.
template <bool DUAL>
__device__ __forceinline__ void produce_groups(const MvParams& p, uint8_t* stages, uint64_t* full, uint64_t* empty,
                                               volatile int* abort_flag, uint32_t mat_off, uint32_t lane) {
    const uint32_t S = p.stages;
    const uint64_t pol = l2_evict_first_policy();
    if (!p.early) pdl_wait();
    uint32_t it = 0;
    for (uint32_t grp = blockIdx.x; grp < p.n_groups; grp += gridDim.x, ++it) {
        const uint32_t s = it % S;
        if (it >= S) {
            bool ok = true;
            if (lane == 0) ok = mbar_wait(&empty[s], ((it / S) - 1u) & 1u, p.err);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok || *abort_flag) {
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
    // drain: no bulk copy may still be landing in this CTA's smem at exit
    if (lane == 0 && *abort_flag) {
        const uint32_t first = it > S ? it - S : 0;
        for (uint32_t j = first; j < it; ++j) mbar_wait(&full[j % S], (j / S) & 1u, p.err);
    }
}

}  // namespace
}  // namespace arc
