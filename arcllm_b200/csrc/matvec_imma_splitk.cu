// Integer-MMA matvec for long rows (K > 3584, e.g. the FFN down projection
// 3584 x 18944): K-chunked stages and a split-K reduction across CTAs.
//
// Work units are (32-row group, chunk of 6 super-blocks); the flattened unit
// list (row-group major) is cut into one contiguous, equal-sized range per
// CTA, so all SMs stream the same number of bytes whatever the row count
// (3584 rows are 112 groups -- no whole-group split balances them over 148
// SMs, but 112 x 13 units do).  A CTA keeps per-row sums in registers while
// consecutive units belong to one row group and leaves a partial when the
// group ends; the CTAs that share a group (at most a few) write their
// partials to a per-device scratch and the last one to arrive adds them in
// CTA order (deterministic) and writes y.
//
// Stages: 32 rows x 6 super-blocks, one 1-D TMA bulk copy per row issued by
// the producer warp's lanes; 12 consumer warps each take one (16-row tile,
// super-block) pair of every unit.  Q6_K rows are not 16-byte aligned (210-byte
// blocks), so each row copy starts at the 16-byte boundary below the row and
// the consumers index from the row's offset inside its slot; the matrix's
// final partial 16 bytes are copied by hand so nothing past the weights is
// read.  x is quantised once per CTA into an image of limb planes for all of K
// (matvec_imma.cuh); warps gather their B fragments per unit.
#include <algorithm>
#include <cmath>
#include <mutex>

#include "arcllm_cuda_internal.h"
#include "common.cuh"
#include "matvec_common.cuh"
#include "matvec_imma.cuh"

namespace arc {
namespace {

constexpr uint32_t kSB = 6;       // super-blocks per unit (even: Q6_K half-block pairing)
constexpr uint32_t kNW = 12;      // consumer warps: (16-row tile m, super-block j) = (w & 1, w >> 1)
constexpr uint32_t kRowsU = 32;   // rows per unit (two 16-row MMA tiles)
constexpr uint32_t kXimSb = 960;  // x image per super-block: 3 x 256 limb bytes + 8 x 6 window floats
constexpr uint32_t kHead = 2 * kMaxStages * 8 + 16;  // full/empty barriers, abort flag (+pad)

struct SplitK {
    float* part;    // [n_rg][slots][32] CTA partials
    uint32_t* cnt;  // [n_rg] arrival counters (zero between launches)
    uint32_t n_ks, n_rg, units, slots, rs;
};

__host__ __device__ inline uint32_t sk_red_off() { return kHead + 32 * 8; }
__host__ __device__ inline uint32_t sk_xim_off(uint32_t S) { return sk_red_off() + 2 * S * kSB * kRowsU * 4; }
__host__ __device__ inline uint32_t sk_stage_off(uint32_t S, uint32_t nb) { return sk_xim_off(S) + nb * kXimSb; }

// CTA that owns unit u when `units` are cut into `grid` contiguous ranges [units*i/grid, units*(i+1)/grid)
__device__ __forceinline__ uint32_t cta_of(uint32_t u, uint32_t units, uint32_t grid) {
    return (uint32_t)((((uint64_t)u + 1) * grid - 1) / units);
}

// Byte offset of row `row`'s chunk inside its 16-byte-aligned copy.
__device__ __forceinline__ uint32_t row_mis(const MvParams& p, uint32_t row, uint32_t sb0, uint32_t bsz) {
    return (uint32_t)(((uint64_t)row * p.rb + (uint64_t)sb0 * bsz) & 15u);
}

template <int FMT>
__device__ __forceinline__ void sk_finish(const MvParams& p, const SplitK& k, const float* red, uint32_t u0,
                                          uint32_t j, uint32_t lane) {
    const uint32_t S = p.stages, s = j % S, par = (j / S) & 1u;
    const uint32_t u = u0 + j, rg = u / k.n_ks;
    const uint32_t rows_g = min(kRowsU, p.rows - rg * kRowsU);
    const float* rs = red + (par * S + s) * kSB * kRowsU;
    const uint32_t first = cta_of(rg * k.n_ks, k.units, gridDim.x);
    const uint32_t last = cta_of(rg * k.n_ks + k.n_ks - 1, k.units, gridDim.x);
    const uint32_t nc = last - first + 1;
    float a = 0.f;
    if (lane < rows_g)
        for (uint32_t j = 0; j < kSB; ++j) a += rs[j * kRowsU + lane];
    const uint32_t row = rg * kRowsU + lane;
    if (nc == 1) {
        if (lane < rows_g) {
            if (p.bias) a += p.bias[row];
            if (p.residual) a = p.residual[row] + a;
            p.y[row] = a;
        }
        return;
    }
    float* slot = k.part + ((uint64_t)rg * k.slots) * kRowsU;
    if (lane < rows_g) slot[(blockIdx.x - first) * kRowsU + lane] = a;
    __threadfence();
    __syncwarp();
    uint32_t old = 0;
    if (lane == 0) old = atomicAdd(&k.cnt[rg], 1u);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old != nc - 1) return;
    __threadfence();  // the last CTA of this row group: add the partials in CTA order
    if (lane < rows_g) {
        const volatile float* vs = slot;
        float t = 0.f;
        for (uint32_t c = 0; c < nc; ++c) t += vs[c * kRowsU + lane];
        if (p.bias) t += p.bias[row];
        if (p.residual) t = p.residual[row] + t;
        p.y[row] = t;
    }
    if (lane == 0) atomicExch(&k.cnt[rg], 0u);
}

template <int FMT>
__global__ void __launch_bounds__((kNW + 1) * 32, 1) matvec_imma_splitk_kernel(const MvParams p, const SplitK k) {
    constexpr uint32_t bsz = FMT == 12 ? 144u : 210u;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kMaxStages;
    volatile int* abort_flag = reinterpret_cast<int*>(empty + kMaxStages);
    double* red_d = reinterpret_cast<double*>(smem + kHead);                // [32]
    float* red = reinterpret_cast<float*>(smem + sk_red_off());            // [2][S][kSB][32]
    uint8_t* xim = smem + sk_xim_off(p.stages);                            // [nb][960]
    uint8_t* stages = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem + sk_stage_off(p.stages, p.nb)) + 127) & ~uintptr_t(127));

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    const uint32_t S = p.stages;
    const uint32_t u0 = (uint32_t)((uint64_t)k.units * blockIdx.x / gridDim.x);
    const uint32_t u1 = (uint32_t)((uint64_t)k.units * (blockIdx.x + 1) / gridDim.x);
    const uint32_t n = u1 - u0;
    pdl_trigger();

    if (tid == kNW * 32) {
        for (uint32_t s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kNW);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();

    // a unit ends this CTA's stretch of its row group: the next unit starts another group, or none follows
    auto ends_group = [&](uint32_t j) { return j + 1 == n || (u0 + j + 1) % k.n_ks == 0; };

    if (warp == kNW) {
        // ---------------- producer ----------------
        const uint64_t pol = l2_evict_first_policy();
        const uint64_t total = (uint64_t)p.rows * p.rb;
        const uint64_t total16 = total & ~(uint64_t)15;
        if (!p.early) pdl_wait();
        uint32_t it = 0;
        bool ok = true;
        auto released = [&](uint32_t j) {
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
            const uint32_t u = u0 + it, rg = u / k.n_ks, ks = u % k.n_ks;
            const uint32_t rows_g = min(kRowsU, p.rows - rg * kRowsU);
            const uint32_t sb0 = ks * kSB, nsb = min(kSB, p.nb - sb0);
            uint8_t* dst = stages + s * p.stage_smem + lane * k.rs;
            // this lane's row: 16-byte-aligned source range [a0, a1), bytes [a1, end) by hand
            uint64_t a0 = 0, a1 = 0, end = 0;
            if (lane < rows_g) {
                const uint64_t src = (uint64_t)(rg * kRowsU + lane) * p.rb + (uint64_t)sb0 * bsz;
                end = src + (uint64_t)nsb * bsz;
                a0 = src & ~(uint64_t)15;
                a1 = max(min((end + 15) & ~(uint64_t)15, total16), a0);
                for (uint64_t b = a1; b < end; ++b) dst[b - a0] = p.w0[b];
            }
            uint32_t bytes = (uint32_t)(a1 - a0);
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) bytes += __shfl_xor_sync(0xffffffffu, bytes, o);
            __syncwarp();
            if (lane == 0) mbar_arrive_expect_tx(&full[s], bytes);
            __syncwarp();
            if (a1 > a0) bulk_g2s(dst, p.w0 + a0, (uint32_t)(a1 - a0), &full[s], pol);
            if (it >= S && ends_group(it - S)) sk_finish<FMT>(p, k, red, u0, it - S, lane);
        }
        if (ok) {
            for (uint32_t j = it > S ? it - S : 0; j < it; ++j) {
                if (!released(j)) {
                    ok = false;
                    break;
                }
                if (ends_group(j)) sk_finish<FMT>(p, k, red, u0, j, lane);
            }
        }
        if (!ok && lane == 0) {  // no bulk copy may still be landing in this CTA's smem at exit
            const uint32_t first = it > S ? it - S : 0;
            for (uint32_t j = first; j < it; ++j) mbar_wait(&full[j % S], (j / S) & 1u, p.err);
        }
        return;
    }

    // ---------------- consumers ----------------
    pdl_wait();  // x, gamma, bias and residual come from the preceding kernels
    const uint32_t jw = lane >> 2, qd = lane & 3u;
    float inv = 1.0f;
    if (p.gamma) {  // fused RMSNorm over all of K
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
    // quantise x into the image, kBatch super-blocks per warp at a time with
    // all their global loads issued before the first is used
    constexpr uint32_t kBatch = 5;
    for (uint32_t sb0w = warp; sb0w < p.nb; sb0w += kBatch * kNW) {
        float4 xa[kBatch][2], ga[kBatch][2];
#pragma unroll
        for (uint32_t b = 0; b < kBatch; ++b) {
            const uint32_t sb = sb0w + b * kNW;
            if (sb < p.nb) {
                const uint32_t e0 = 256u * sb + 32u * jw + 8u * qd;
                xa[b][0] = *reinterpret_cast<const float4*>(p.x + e0);
                xa[b][1] = *reinterpret_cast<const float4*>(p.x + e0 + 4);
                if (p.gamma) {
                    ga[b][0] = *reinterpret_cast<const float4*>(p.gamma + e0);
                    ga[b][1] = *reinterpret_cast<const float4*>(p.gamma + e0 + 4);
                }
            }
        }
#pragma unroll
        for (uint32_t b = 0; b < kBatch; ++b) {
            const uint32_t sb = sb0w + b * kNW;
            if (sb >= p.nb) break;  // warp-uniform
            float v[8] = {xa[b][0].x, xa[b][0].y, xa[b][0].z, xa[b][0].w, xa[b][1].x, xa[b][1].y, xa[b][1].z, xa[b][1].w};
            if (p.gamma) {
                const float gv[8] = {ga[b][0].x, ga[b][0].y, ga[b][0].z, ga[b][0].w,
                                     ga[b][1].x, ga[b][1].y, ga[b][1].z, ga[b][1].w};
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = (v[i] * inv) * gv[i];
            }
            uint8_t* img = xim + sb * kXimSb;
            quantize8<FMT>(v, lane, img, reinterpret_cast<float*>(img + 768));
        }
    }
    named_bar_sync(1, kNW * 32u);  // the whole x image is in place

    const uint32_t g = lane >> 2, t = lane & 3u;
    const uint32_t m = warp & 1u, j = warp >> 1;  // this warp's 16-row tile and super-block of every unit
    // tile rows (lanes g, lanes g+8): Q6_K takes rows 4g+m and 4g+2+m so each LDS sees one skew (conflict-free)
    const uint32_t ra = FMT == 14 ? 4u * g + m : 16u * m + g;
    const uint32_t rb2 = FMT == 14 ? 4u * g + 2u + m : 16u * m + g + 8u;
    float y0 = 0.f, y1 = 0.f;
    for (uint32_t it = 0; it < n; ++it) {
        const uint32_t s = it % S;
        if (!mbar_wait(&full[s], (it / S) & 1u, p.err)) *abort_flag = 1;
        if (*abort_flag) break;
        const uint32_t u = u0 + it, rg = u / k.n_ks, ks = u % k.n_ks;
        const uint32_t sb0 = ks * kSB, nsb = min(kSB, p.nb - sb0);
        const uint8_t* st = stages + s * p.stage_smem;
        if (j < nsb) {
            const uint32_t sbA = sb0 + j, sbB = FMT == 14 ? sb0 + (j ^ 1u) : sbA;
            const uint8_t* iA = xim + sbA * kXimSb;
            const uint8_t* iB = xim + sbB * kXimSb;
            XFrag f;
            gather_xfrag<FMT>(iA, reinterpret_cast<const float*>(iA + 768), iB,
                              reinterpret_cast<const float*>(iB + 768), lane, f);
            const uint32_t row0 = ra * k.rs + row_mis(p, rg * kRowsU + ra, sb0, bsz);
            const uint32_t row1 = rb2 * k.rs + row_mis(p, rg * kRowsU + rb2, sb0, bsz);
            if (FMT == 12)
                q4_tile(st, row0 + j * bsz, row1 + j * bsz, t, f, y0, y1);
            else if (j & 1u)
                q6_tile<true>(st, row0, row1, j * bsz, (j ^ 1u) * bsz, t, f, y0, y1);
            else
                q6_tile<false>(st, row0, row1, j * bsz, (j ^ 1u) * bsz, t, f, y0, y1);
        }
        if (ends_group(it)) {
            // hand this warp's row sums to the producer (slot of this stage round, column j) and restart
            float* rs = red + (((it / S) & 1u) * S + s) * kSB * kRowsU + j * kRowsU;
            y0 += __shfl_xor_sync(0xffffffffu, y0, 1);
            y0 += __shfl_xor_sync(0xffffffffu, y0, 2);
            y1 += __shfl_xor_sync(0xffffffffu, y1, 1);
            y1 += __shfl_xor_sync(0xffffffffu, y1, 2);
            if (t == 0) {
                rs[ra] = y0;
                rs[rb2] = y1;
            }
            y0 = y1 = 0.f;
        }
        __syncwarp();
        if (lane == 0) {
            __threadfence_block();
            mbar_arrive(&empty[s]);
        }
    }
}

struct SkScratch {
    float* part = nullptr;
    uint32_t* cnt = nullptr;
    size_t part_floats = 0, cnt_n = 0;
};
std::mutex g_sk_mutex;
SkScratch g_sk[64];

struct SkConfig {
    uint32_t S, rs, stage_smem, smem, grid;
    SplitK k;
};

SkConfig sk_config(int fmt, uint32_t rows, uint32_t kk, int sms) {
    SkConfig c{};
    const uint32_t nb = kk / 256u;
    const uint32_t bsz = fmt == 12 ? 144u : 210u;
    // row slot stride: Q4_K 8 words mod 32 banks (LDS.64 half-warps conflict-free); Q6_K room for the
    // 16-byte skew and 16 x odd mod 128 bytes, so 8 rows of one residue mod 4 (one skew) hit distinct banks
    uint32_t rs = (kSB * bsz + (fmt == 12 ? 0u : 12u) + 15u) & ~15u;
    while (fmt == 12 ? ((rs / 4u) % 32u != 8u) : ((rs % 128u) / 16u % 2u != 1u)) rs += 16u;
    c.rs = rs;
    c.stage_smem = kRowsU * c.rs;
    c.k.n_ks = (nb + kSB - 1) / kSB;
    c.k.n_rg = (rows + kRowsU - 1) / kRowsU;
    c.k.units = c.k.n_ks * c.k.n_rg;
    c.k.rs = c.rs;
    c.grid = std::min<uint32_t>(c.k.units, (uint32_t)sms);
    // contributors per row group: CTAs whose unit range meets it
    uint32_t slots = 1;
    for (uint32_t rg = 0; rg < c.k.n_rg; ++rg) {
        const uint64_t fu = (uint64_t)rg * c.k.n_ks, lu = fu + c.k.n_ks - 1;
        const uint32_t a = (uint32_t)(((fu + 1) * c.grid - 1) / c.k.units);
        const uint32_t b = (uint32_t)(((lu + 1) * c.grid - 1) / c.k.units);
        slots = std::max(slots, b - a + 1);
    }
    c.k.slots = slots;
    const uint32_t budget = 227u * 1024u;
    uint32_t S = kMaxStages;
    while (S > 2 && sk_stage_off(S, nb) + 128u + S * c.stage_smem > budget) --S;
    c.S = S;
    c.smem = sk_stage_off(S, nb) + 128u + S * c.stage_smem;
    return c;
}

int sk_sm_count() {
    static int sm_count[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    int& sms = sm_count[dev & 63];
    if (sms <= 0 && cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) sms = 148;
    return sms;
}

}  // namespace

int matvec_splitk_reserve(int fmt, uint32_t rows, uint32_t k) {
    const SkConfig c = sk_config(fmt, rows, k, sk_sm_count());
    const size_t need_part = (size_t)c.k.n_rg * c.k.slots * kRowsU, need_cnt = c.k.n_rg;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(g_sk_mutex);
    SkScratch& sc = g_sk[dev & 63];
    if (sc.part_floats >= need_part && sc.cnt_n >= need_cnt) return ARC_OK;
    const size_t np = std::max(need_part, sc.part_floats), nc = std::max(need_cnt, sc.cnt_n);
    float* part = nullptr;
    uint32_t* cnt = nullptr;
    cudaError_t e = cudaMalloc(&part, np * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&cnt, nc * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMemset(cnt, 0, nc * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaFree(part);
        cudaFree(cnt);
        return set_cuda_error(e, "matvec split-K scratch");
    }
    cudaFree(sc.part);  // grown only outside concurrent use (documented)
    cudaFree(sc.cnt);
    sc.part = part;
    sc.cnt = cnt;
    sc.part_floats = np;
    sc.cnt_n = nc;
    return ARC_OK;
}

int matvec_splitk_prepare() {
    static bool done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (done[dev & 63]) return ARC_OK;
    cudaError_t e = cudaFuncSetAttribute(matvec_imma_splitk_kernel<12>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         227 * 1024);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(matvec_imma_splitk_kernel<14>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 227 * 1024);
    if (e != cudaSuccess) return set_cuda_error(e, "matvec split-K prepare");
    done[dev & 63] = true;
    return ARC_OK;
}

// Single matrix, K > 3584 with an even number of super-blocks (Q6_K pairing;
// Q4_K too, so that both formats take the same path), the x image in smem.
bool matvec_splitk_supported(int fmt, bool dual, uint32_t rows, uint32_t k) {
    if ((fmt != 12 && fmt != 14) || dual || rows == 0 || k % 512u) return false;
    const uint32_t nb = k / 256u;
    if (nb <= 14) return false;
    return sk_config(fmt, rows, k, 148).smem <= 227u * 1024u;
}

int matvec_splitk_launch(int fmt, const void* w, uint32_t rows, uint32_t k, const float* x, const float* gamma,
                         float eps, const float* bias, const float* residual, float* y, cudaStream_t stream) {
    if (!matvec_splitk_supported(fmt, false, rows, k))
        return set_error(ARC_E_UNSUPPORTED_SHAPE, "matvec split-K: shape not supported");
    if (!w || !x || !y) return set_error(ARC_E_INVALID_ARGUMENT, "matvec: null pointer");
    if (reinterpret_cast<uintptr_t>(w) & 15u)
        return set_error(ARC_E_ALIGNMENT, "matvec: weight pointers must be 16-byte aligned");
    int st = matvec_splitk_prepare();
    if (st == ARC_OK) st = matvec_splitk_reserve(fmt, rows, k);
    if (st != ARC_OK) return st;
    const SkConfig c = sk_config(fmt, rows, k, sk_sm_count());
    int dev = 0;
    cudaGetDevice(&dev);
    SplitK sk = c.k;
    {
        std::lock_guard<std::mutex> lock(g_sk_mutex);
        sk.part = g_sk[dev & 63].part;
        sk.cnt = g_sk[dev & 63].cnt;
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
    p.k = k;
    p.nb = k / 256u;
    p.rb = p.nb * (fmt == 12 ? 144u : 210u);
    p.G = kRowsU;
    p.n_groups = c.k.n_rg;
    p.stages = c.S;
    p.stage_smem = c.stage_smem;
    p.early = pdl_enabled() ? 1u : 0u;
    const cudaError_t e =
        fmt == 12 ? launch_kernel(matvec_imma_splitk_kernel<12>, dim3(c.grid), dim3((kNW + 1) * 32), c.smem, stream, p, sk)
                  : launch_kernel(matvec_imma_splitk_kernel<14>, dim3(c.grid), dim3((kNW + 1) * 32), c.smem, stream, p, sk);
    return e == cudaSuccess ? ARC_OK : set_cuda_error(e, "matvec split-K launch");
}

}  // namespace arc
