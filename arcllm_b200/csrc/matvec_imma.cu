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
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>

#include "arcllm_cuda_internal.h"
#include "common.cuh"
#include "matvec_common.cuh"
#include "matvec_imma.cuh"

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

// Final row sums of one finished stage round `itr`: the consumer warps' partials
// (red[parity][slot][warp][row]) added in warp order, plus bias / residual or
// the SiLU(gate)*up product, written to y.  Run by the producer warp.
template <int G, bool DUAL>
__device__ __forceinline__ void finish_rows(const MvParams& p, const float* red, uint32_t nwc, uint32_t itr,
                                            uint32_t lane) {
    constexpr int NV = DUAL ? 2 * G : G;
    const uint32_t S = p.stages, s = itr % S, par = (itr / S) & 1u;
    const uint32_t grp = job_cta(p) + itr * job_ctas(p);
    const uint32_t rows_g = min(p.G, p.rows - grp * p.G);
    const float* rs = red + (par * S + s) * nwc * NV;
    for (uint32_t r = lane; (DUAL || p.rope_mode == 0) && r < rows_g; r += 32u) {
        const uint32_t row = grp * p.G + r;
        float a = 0.f;
        for (uint32_t w = 0; w < nwc; ++w) a += rs[w * NV + r];
        if (DUAL) {
            float u = 0.f;
            for (uint32_t w = 0; w < nwc; ++w) u += rs[w * NV + G + r];
            // src/p8c_segmented_access_correctness.cpp:1064-1073 (silu(g)*u)
            p.y[row] = (a / (1.0f + expf(-a))) * u;
        } else if (p.rope_mode == 0) {
            if (p.bias) a += p.bias[row];
            if (p.residual) a = p.residual[row] + a;
            p.y[row] = a;
            if (p.n_ranks) {  // all-gather: the row, tagged with the epoch, into every rank's word array
                const unsigned long long word = ((unsigned long long)p.epoch << 32) | __float_as_uint(a);
#pragma unroll
                for (uint32_t q = 0; q < kMaxRanks; ++q)
                    if (q < p.n_ranks) st_relaxed_sys_u64(p.gather_ll[q] + p.gather_row0 + row, word);
            }
        }
    }
    if (!DUAL && p.rope_mode != 0) {
        // fused RoPE / fp16 KV store: one row per lane (G <= 32), rotation pairs (2p, 2p+1) in
        // neighbouring lanes; the same operations as the standalone rope_kv_store kernel
        const uint32_t row = grp * p.G + lane;
        const bool act = lane < rows_g;
        float a = 0.f;
        if (act) {
            for (uint32_t w = 0; w < nwc; ++w) a += rs[w * NV + lane];
            if (p.bias) a += p.bias[row];
        }
        const uint32_t pos = *p.rope_pos;
        const bool pos_ok = pos < p.max_ctx;
        if (!pos_ok && lane == 0) raise_error(p.err, ARC_DEV_ERR_BOUNDS);
        float v = a;
        if (p.rope_mode <= 2u) {
            const float b = __shfl_xor_sync(0xffffffffu, a, 1);
            const float2 cs = pos_ok ? p.rope_table[(uint64_t)pos * p.rope_half + (row >> 1) % p.rope_half]
                                     : make_float2(1.f, 0.f);
            v = (row & 1u) ? __fadd_rn(__fmul_rn(b, cs.y), __fmul_rn(a, cs.x))
                           : __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
        }
        if (act) {
            p.y[row] = v;
            if (p.rope_mode >= 2u && pos_ok) p.cache[(uint64_t)pos * p.rows + row] = __half_as_ushort(__float2half_rn(v));
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
// End of the rank all-gather, run by every thread of each CTA once the CTA's
// own rows are stored: CTA b takes an equal slice [i0, i1) of the whole
// result, reads this rank's words of the slice (up to four per thread in
// flight) until each carries this launch's epoch and writes the values to
// gather_out.  The words come from every rank's CTAs, so the launch ends once
// the last row of the slowest rank has landed -- no fence, counter or flag:
// each 64-bit word is its own flag.  Gives up after p.wait_ns with
// ARC_DEV_ERR_TIMEOUT.
__device__ __forceinline__ void gather_collect(const MvParams& p) {
    const uint32_t n = p.gather_rows_total, per = (n + gridDim.x - 1u) / gridDim.x;
    const uint32_t i0 = blockIdx.x * per, i1 = min(n, i0 + per), nt = blockDim.x;
    const unsigned long long t0 = globaltimer();
    for (uint32_t base = i0 + threadIdx.x; base < i1; base += 4u * nt) {
        unsigned long long v[4];
#pragma unroll
        for (uint32_t j = 0; j < 4; ++j)
            if (base + j * nt < i1) v[j] = ld_relaxed_sys_u64(p.gather_own + base + j * nt);
#pragma unroll
        for (uint32_t j = 0; j < 4; ++j) {
            const uint32_t i = base + j * nt;
            if (i >= i1) break;
            while ((uint32_t)(v[j] >> 32) != p.epoch) {
                if (globaltimer() - t0 > p.wait_ns) {
                    raise_error(p.err, ARC_DEV_ERR_TIMEOUT);
                    return;
                }
                __nanosleep(32);
                v[j] = ld_relaxed_sys_u64(p.gather_own + i);
            }
            p.gather_out[i] = __uint_as_float((uint32_t)v[j]);
        }
    }
}

template <int G, bool DUAL>
__device__ __forceinline__ void produce_and_finish(const MvParams& p, uint8_t* stages, uint64_t* full,
                                                   uint64_t* empty, volatile int* abort_flag, uint32_t mat_off,
                                                   const float* red, uint32_t nwc, uint32_t lane) {
    const uint32_t S = p.stages;
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
    for (uint32_t grp = job_cta(p); grp < p.n_groups; grp += job_ctas(p), ++it) {
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
        if (it == S && p.early) pdl_wait();  // the epilogue reads predecessors' outputs (bias, residual, position)
        if (it >= S) finish_rows<G, DUAL>(p, red, nwc, it - S, lane);
    }
    if (ok) {
        if (it <= S && p.early) pdl_wait();
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

// The consumer warps of matvec_imma_kernel.
template <int FMT, int MT, bool DUAL>
__device__ __forceinline__ void consume(const MvParams& p, const uint8_t* stages, uint64_t* full, uint64_t* empty,
                                        volatile int* abort_flag, float* red, double* red_d, uint8_t* xscr,
                                        uint32_t nwc, uint32_t warp, uint32_t lane) {
    constexpr int G = 16 * MT;
    constexpr int NV = DUAL ? 2 * G : G;
    const uint32_t S = p.stages;
    const uint32_t mat_off = p.G * p.rb;

    // Q4_K: warp w owns super-block w.  Q6_K: half 0 of block w and half 1 of
    // block w^1 (K has an even number of blocks), see q6_tile.
    const uint32_t bA = warp, bB = (FMT == 14) ? (warp ^ 1u) : warp;
    XFrag f;
    pdl_wait();  // x and gamma come from the preceding kernels
    build_xfrag<FMT>(p.x, p.gamma, p.eps, p.k, red_d, nwc, warp, bA, bB, lane, xscr + warp * kXScratch, f);
    const uint32_t g = lane >> 2, t = lane & 3u;
    const uint32_t bsz = FMT == 12 ? 144u : 210u;
    const uint32_t offA = bA * bsz, offB = bB * bsz;
    const bool oddA = FMT == 14 && (offA & 3u) != 0u;

    uint32_t it = 0;
    for (uint32_t grp = job_cta(p); grp < p.n_groups; grp += job_ctas(p), ++it) {
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

// One CTA of a whole-row matvec: barriers, then the producer warp and the
// consumer warps (and, with n_ranks, the all-gather collect).
template <int FMT, int MT, bool DUAL>
__device__ __forceinline__ void imma_cta(const MvParams& p, uint32_t nwc) {
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
    uint8_t* stages = smem_align_up<128>(smem, imma_stage_off(p.stages, nwc, NV));

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    const uint32_t NT = nwc * 32u;
    const uint32_t S = p.stages;
    const uint32_t mat_off = p.G * p.rb;
    pdl_trigger();

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
    } else {
        consume<FMT, MT, DUAL>(p, stages, full, empty, abort_flag, red, red_d, xscr, nwc, warp, lane);
    }
    if constexpr (!DUAL) {
        if (p.n_ranks) {
            __syncthreads();  // the producer has stored this CTA's rows
            if (!*abort_flag) gather_collect(p);
        }
    }
}

template <int FMT, int MT, bool DUAL>
__global__ void __launch_bounds__(15 * 32, 1) matvec_imma_kernel(const MvParams p, uint32_t nwc) {
    imma_cta<FMT, MT, DUAL>(p, nwc);
}

// Up to three independent single-matrix jobs with the same K in one launch
// (the decode step's Q, K and V projections: they read the same x, and one
// grid lets the next kernel follow with programmatic dependent launch instead
// of after a join of streams).  Job j owns CTAs [pj.cta0, pj.cta0 + pj.ncta);
// fj is its format (12 Q4_K, 14 Q6_K).
// Dynamic shared memory of the multi-job kernel: 227 KB less room for its static copy of a job's parameters.
constexpr uint32_t kMultiMaxDynSmem = 227u * 1024u - 1024u;

// The CTA copies its job's parameters into shared memory first, so the kernel
// holds one body per format instead of one per (job, format): each CTA runs
// its code once, and a smaller kernel means fewer cold instruction fetches.
__global__ void __launch_bounds__(15 * 32, 1)
    matvec_imma_multi_kernel(const __grid_constant__ MvParams p0, const __grid_constant__ MvParams p1,
                             const __grid_constant__ MvParams p2, int f0, int f1, int f2, uint32_t nwc) {
    __shared__ __align__(16) MvParams sp;
    static_assert(sizeof(MvParams) % 4 == 0, "copied as words");
    const uint32_t job = blockIdx.x < p1.cta0 ? 0u : blockIdx.x < p2.cta0 ? 1u : 2u;
    const uint32_t* src = reinterpret_cast<const uint32_t*>(job == 0 ? &p0 : job == 1 ? &p1 : &p2);
    for (uint32_t i = threadIdx.x; i < sizeof(MvParams) / 4; i += blockDim.x)
        reinterpret_cast<uint32_t*>(&sp)[i] = src[i];
    __syncthreads();
    if ((job == 0 ? f0 : job == 1 ? f1 : f2) == 12)
        imma_cta<12, 2, false>(sp, nwc);
    else
        imma_cta<14, 2, false>(sp, nwc);
}

template <int FMT, int MT, bool DUAL>
cudaError_t launch_imma_t(const MvParams& p, uint32_t nwc, uint32_t smem, uint32_t grid, cudaStream_t st) {
    return launch_kernel(matvec_imma_kernel<FMT, MT, DUAL>, dim3(grid), dim3((nwc + 1) * 32), smem, st, p, nwc);
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
    static std::atomic<bool> done[64] = {};  // concurrent first calls set the same (idempotent) attributes
    const int slot = device_slot();
    if (slot < 0) return set_error(ARC_E_CUDA, "matvec_imma prepare: no current device below index 64");
    if (done[slot].load(std::memory_order_acquire)) return ARC_OK;
    cudaError_t e = set_attr_imma<12, 1, false>();
    if (e == cudaSuccess) e = set_attr_imma<12, 2, false>();
    if (e == cudaSuccess) e = set_attr_imma<12, 1, true>();
    if (e == cudaSuccess) e = set_attr_imma<12, 2, true>();
    if (e == cudaSuccess) e = set_attr_imma<14, 1, false>();
    if (e == cudaSuccess) e = set_attr_imma<14, 2, false>();
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(matvec_imma_multi_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 kMultiMaxDynSmem);
    if (e != cudaSuccess) return set_cuda_error(e, "matvec_imma prepare");
    done[slot].store(true, std::memory_order_release);
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

namespace {
// Parameters of one whole-row launch (matvec_imma_supported already checked).
int imma_params(int fmt, bool dual, const void* w0, const void* w1, uint32_t rows, uint32_t k, const float* x,
                const float* gamma, float eps, const float* bias, const float* residual, float* y,
                const RopeEpilogue* rope, const RankGather* gather, MvParams& p, ImmaConfig& c) {
    if (!w0 || !x || !y || (dual && !w1)) return set_error(ARC_E_INVALID_ARGUMENT, "matvec: null pointer");
    if ((reinterpret_cast<uintptr_t>(w0) & 15u) || (w1 && (reinterpret_cast<uintptr_t>(w1) & 15u)))
        return set_error(ARC_E_ALIGNMENT, "matvec: weight pointers must be 16-byte aligned");
    c = imma_config(fmt, dual, k);
    const uint32_t nb = k / 256u;
    p = MvParams{};
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
    p.early = pdl_enabled() ? 1u : 0u;
    if (rope && rope->mode != 0) {
        if (dual || residual || rope->mode > 3u || rope->half == 0 || (rows % (2u * rope->half)) != 0u || !rope->pos ||
            (rope->mode <= 2u && !rope->table) || (rope->mode >= 2u && !rope->cache))
            return set_error(ARC_E_INVALID_ARGUMENT, "matvec_imma: bad fused RoPE epilogue");
        p.rope_mode = rope->mode;
        p.rope_half = rope->half;
        p.rope_table = rope->table;
        p.rope_pos = rope->pos;
        p.cache = rope->cache;
        p.max_ctx = rope->max_ctx;
    }
    if (gather && gather->n_ranks != 0) {
        if (dual || (rope && rope->mode != 0) || gather->n_ranks > kMaxRanks || gather->self_rank >= gather->n_ranks ||
            !gather->out || gather->epoch == 0 || (uint64_t)gather->row0 + rows > gather->rows_total)
            return set_error(ARC_E_INVALID_ARGUMENT, "matvec_imma: bad rank all-gather epilogue");
        p.n_ranks = gather->n_ranks;
        p.self_rank = gather->self_rank;
        p.epoch = gather->epoch;
        p.wait_ns = gather->wait_ns;
        for (uint32_t r = 0; r < gather->n_ranks; ++r) {
            if (!gather->ll[r] || (reinterpret_cast<uintptr_t>(gather->ll[r]) & 7u))
                return set_error(ARC_E_INVALID_ARGUMENT, "matvec_imma: null or unaligned rank word array");
            p.gather_ll[r] = gather->ll[r];
        }
        p.gather_own = gather->ll[gather->self_rank];
        p.gather_out = gather->out;
        p.gather_row0 = gather->row0;
        p.gather_rows_total = gather->rows_total;
    }
    return ARC_OK;
}

uint32_t imma_sm_count() {
    static std::atomic<int> sm_count[64] = {};  // per device, queried once
    const int slot = device_slot();
    int sms = slot >= 0 ? sm_count[slot].load(std::memory_order_relaxed) : 0;
    if (sms > 0) return (uint32_t)sms;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
        sms = 148;
    if (slot >= 0) sm_count[slot].store(sms, std::memory_order_relaxed);
    return (uint32_t)sms;
}
}  // namespace

int matvec_imma_launch(int fmt, bool dual, const void* w0, const void* w1, uint32_t rows, uint32_t k, const float* x,
                       const float* gamma, float eps, const float* bias, const float* residual, float* y,
                       cudaStream_t stream, const RopeEpilogue* rope, const RankGather* gather) {
    if (!matvec_imma_supported(fmt, dual, rows, k))
        return set_error(ARC_E_UNSUPPORTED_SHAPE, "matvec_imma: shape outside K/256 <= 14 (even for Q6_K)");
    int st = matvec_imma_prepare();
    if (st != ARC_OK) return st;
    MvParams p;
    ImmaConfig c;
    st = imma_params(fmt, dual, w0, w1, rows, k, x, gamma, eps, bias, residual, y, rope, gather, p, c);
    if (st != ARC_OK) return st;
    const uint32_t nb = k / 256u;
    const uint32_t grid = std::min(p.n_groups, imma_sm_count());
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

// Three whole-row jobs sharing x, gamma and K in one grid (matvec_imma_multi_kernel): each
// job gets one CTA per row group, so all groups of all jobs must fit on the SMs at once and
// every job must use 32-row groups.
bool matvec_imma_multi_supported(const ImmaJob (&jobs)[3], uint32_t k) {
    uint32_t ctas = 0;
    for (const ImmaJob& j : jobs) {
        if (!matvec_imma_supported(j.fmt, false, j.rows, k)) return false;
        const ImmaConfig c = imma_config(j.fmt, false, k);
        // 32-row groups; the job's shared memory plus the kernel's copy of its parameters fits
        if (c.MT != 2 || c.smem > kMultiMaxDynSmem) return false;
        ctas += (j.rows + c.G - 1u) / c.G;
    }
    return ctas <= imma_sm_count();
}

int matvec_imma_multi_launch(const ImmaJob (&jobs)[3], uint32_t k, const float* x, const float* gamma, float eps,
                             cudaStream_t stream) {
    if (!matvec_imma_multi_supported(jobs, k))
        return set_error(ARC_E_UNSUPPORTED_SHAPE, "matvec_imma multi: jobs do not fit one grid");
    int st = matvec_imma_prepare();
    if (st != ARC_OK) return st;
    MvParams p[3];
    uint32_t cta = 0, smem = 0;
    for (int i = 0; i < 3; ++i) {
        const ImmaJob& j = jobs[i];
        ImmaConfig c;
        st = imma_params(j.fmt, false, j.w, nullptr, j.rows, k, x, gamma, eps, j.bias, nullptr, j.y, j.rope, nullptr,
                         p[i], c);
        if (st != ARC_OK) return st;
        p[i].cta0 = cta;
        p[i].ncta = p[i].n_groups;
        cta += p[i].ncta;
        smem = std::max(smem, c.smem);
    }
    const uint32_t nwc = k / 256u;  // one consumer warp per super-block, plus the producer warp
    const cudaError_t e = launch_kernel(matvec_imma_multi_kernel, dim3(cta), dim3((nwc + 1) * 32), smem, stream, p[0],
                                        p[1], p[2], jobs[0].fmt, jobs[1].fmt, jobs[2].fmt, nwc);
    if (e != cudaSuccess) return set_cuda_error(e, "matvec_imma multi launch");
    return ARC_OK;
}

}  // namespace arc
