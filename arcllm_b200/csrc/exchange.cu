// Rank exchange over NVLink peer stores: the cross-rank steps of the
// tensor-parallel decode (generate() sharded over the GPUs of one node) and of
// the row-sharded matvecs.
//
// The reference decodes on one device (src/arcllm_v1_runtime.cpp:371-421, one
// Vulkan queue, src/arcllm_v1_vulkan_runtime_support.h:535).  Sharded over N
// GPUs, the FFN gate/up rows and the matching K window of the FFN down
// projection are split over the ranks, so the down projection's partial sums
// (3584 floats at the Qwen2.5-7B shape) are all-reduced on every rank (the
// reduce form), and the LM-head rows are split, so the ranks' greedy-selection
// records (4 words each) are all-gathered (the gather form, which also
// re-assembles row-sharded matvec outputs).
//
// exchange_kernel runs kExCtas CTAs of 128 threads per rank.  Every 32-bit
// word of this rank's slice (or, in the reduce form, of its whole partial
// vector, into slot `rank`) is stored into every rank's exchange buffer as ONE
// 64-bit word (seq << 32 | value) -- its own buffer with local stores, the
// others with NVLink peer stores; stores only, nothing reads another GPU's
// memory.  Then each CTA reads its share of the assembled vector out of its
// own buffer, waiting (bounded by %globaltimer) until each word carries this
// exchange's sequence number, and writes the values to `dst` (reduce form: the
// ranks' slots added in rank order, plus an optional residual -- the
// all-reduce of the K-sharded FFN down projection).  Every word is its own
// flag, so no fence and no separate flag handshake is needed.
//
// Buffer of one rank (W = the largest vector's word count rounded up to 4):
//   [0, 2W) 64-bit words   two data regions, picked by the parity of the sequence number
//   then kExCtas u32       the per-CTA sequence counters of this rank (local; CTA b
//                          advances counter b by one per exchange)
// Every rank runs the same exchanges in the same order (the decode graph) with
// the same fixed grid, so all counters agree without host involvement and a
// graph replays unchanged.  Why two regions suffice: a rank can store into a
// peer's region of sequence e+2 only after its own exchange e+1 completed,
// which needed that peer's e+1 words, which the peer stores only after its
// exchange e (which reads the same region) completed -- the exchanges of one
// rank are stream ordered.  A word of an older exchange in the same region
// carries an older sequence number and is never taken for a newer one.  A
// wait that runs out sets the device error word's timeout bit and returns;
// the ranks may then disagree, so the exchange buffers must be re-created
// (zeroed) before further use.
#include "arcllm_cuda_internal.h"
#include "common.cuh"
#include "decode_ops.h"

namespace arc {
namespace {

constexpr uint32_t kMaxExRanks = 8;
constexpr uint32_t kExCtas = 16;

struct ExParams {
    unsigned long long* data[kMaxExRanks];  // rank q's word regions, as this process maps them
    uint32_t* seq;                          // this rank's per-CTA counters [kExCtas]
    const uint32_t* src;                    // this rank's slice
    uint32_t* dst;                          // the assembled vector (n_total words)
    uint32_t W, n_local, off, n_total, n_ranks, rank;
    unsigned long long wait_ns;
    unsigned int* err;
    // reduce form: every rank contributes a whole n_total-float vector (slot `rank` of the
    // region) and dst = residual (nullable) + the slots added in rank order
    uint32_t reduce;
    const float* residual;
};

// 128 threads of at most 32 registers: 4096 registers, which fit beside one CTA
// of the matvec kernels (480 threads x <= 128 registers), so the exchange CTAs
// are resident -- launched early by programmatic dependent launch, parked in
// griddepcontrol.wait -- when the kernel producing the slice ends.
constexpr uint32_t kExThreads = 128;

// Wait until word i of the own region carries `tag` (bounded); false on timeout.
__device__ __forceinline__ bool await_word(const unsigned long long* own, uint32_t i, uint32_t tag,
                                           unsigned long long& v, unsigned long long t0, const ExParams& p) {
    while ((uint32_t)(v >> 32) != tag) {
        if (globaltimer() - t0 > p.wait_ns) {
            raise_error(p.err, ARC_DEV_ERR_TIMEOUT);
            return false;
        }
        __nanosleep(32);
        v = ld_relaxed_sys_u64(own + i);
    }
    return true;
}

__global__ void __launch_bounds__(kExThreads, 16) exchange_kernel(const ExParams p) {
    __shared__ uint32_t s_seq;
    pdl_trigger();
    pdl_wait();  // the slice comes from the preceding kernel
    const uint32_t tid = threadIdx.x, nthr = gridDim.x * blockDim.x, gtid = blockIdx.x * blockDim.x + tid;
    if (tid == 0) {  // counter b is read and advanced only by CTA b of each exchange, in stream order
        s_seq = *reinterpret_cast<volatile uint32_t*>(p.seq + blockIdx.x) + 1u;
        p.seq[blockIdx.x] = s_seq;
    }
    __syncthreads();
    const uint32_t seq = s_seq, region = (seq & 1u) * p.W;
    const unsigned long long tag = (unsigned long long)seq << 32;
    for (uint32_t i = gtid; i < p.n_local; i += nthr) {
        const unsigned long long w = tag | p.src[i];
#pragma unroll
        for (uint32_t q = 0; q < kMaxExRanks; ++q)
            if (q < p.n_ranks) st_relaxed_sys_u64(p.data[q] + region + p.off + i, w);
    }
    const unsigned long long* own = p.data[0];
#pragma unroll
    for (uint32_t q = 1; q < kMaxExRanks; ++q)
        if (q == p.rank) own = p.data[q];
    own += region;
    const unsigned long long t0 = globaltimer();
    if (p.reduce) {  // the same sum, in the same order, on every rank
        float* out = reinterpret_cast<float*>(p.dst);
        for (uint32_t i = gtid; i < p.n_total; i += nthr) {
            unsigned long long v[kMaxExRanks];
#pragma unroll
            for (uint32_t q = 0; q < kMaxExRanks; ++q)  // every slot's word in flight before the first wait
                if (q < p.n_ranks) v[q] = ld_relaxed_sys_u64(own + (uint64_t)q * p.n_total + i);
            float t = 0.f;
#pragma unroll
            for (uint32_t q = 0; q < kMaxExRanks; ++q) {
                if (q >= p.n_ranks) break;
                if (!await_word(own, q * p.n_total + i, seq, v[q], t0, p)) return;
                const float f = __uint_as_float((uint32_t)v[q]);
                t = q ? t + f : f;
            }
            out[i] = p.residual ? p.residual[i] + t : t;
        }
        return;
    }
    for (uint32_t base = gtid; base < p.n_total; base += 4u * nthr) {
        unsigned long long v[4];
#pragma unroll
        for (uint32_t j = 0; j < 4; ++j)
            if (base + j * nthr < p.n_total) v[j] = ld_relaxed_sys_u64(own + base + j * nthr);
#pragma unroll
        for (uint32_t j = 0; j < 4; ++j) {
            const uint32_t i = base + j * nthr;
            if (i >= p.n_total) break;
            if (!await_word(own, i, seq, v[j], t0, p)) return;
            p.dst[i] = (uint32_t)v[j];
        }
    }
}

// Data regions are whole 32-byte units.
inline uint32_t region_words(uint32_t max_words) { return (max_words + 3u) & ~3u; }

}  // namespace

uint64_t exchange_buffer_bytes(uint32_t max_words) {
    return ((uint64_t)2u * region_words(max_words) * 8u + kExCtas * 4u + 255u) / 256u * 256u;
}

namespace {
int exchange_launch(const ExchangeRanks& ex, const void* src, uint32_t n_local, uint32_t off, void* dst,
                    uint32_t n_total, const float* residual, bool reduce, cudaStream_t stream) {
    if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 3u)
        return set_error(ARC_E_ALIGNMENT, "exchange: src and dst must be 4-byte aligned");
    ExParams p{};
    for (uint32_t q = 0; q < ex.n_ranks; ++q) {
        if (!ex.bufs[q] || (reinterpret_cast<uintptr_t>(ex.bufs[q]) & 255u))
            return set_error(ARC_E_ALIGNMENT, "exchange: rank buffers must be non-null and 256-byte aligned");
        p.data[q] = static_cast<unsigned long long*>(ex.bufs[q]);
    }
    p.seq = reinterpret_cast<uint32_t*>(p.data[ex.rank] + 2u * region_words(ex.max_words));
    p.src = static_cast<const uint32_t*>(src);
    p.dst = static_cast<uint32_t*>(dst);
    p.W = region_words(ex.max_words);
    p.n_local = n_local;
    p.off = off;
    p.n_total = n_total;
    p.n_ranks = ex.n_ranks;
    p.rank = ex.rank;
    p.wait_ns = (unsigned long long)(ex.timeout_us ? ex.timeout_us : 2000000u) * 1000ull;
    p.err = dev_error_word();
    p.reduce = reduce ? 1u : 0u;
    p.residual = residual;
    return launch_checked(launch_kernel(exchange_kernel, dim3(kExCtas), dim3(kExThreads), 0, stream, p),
                          "exchange launch");
}
}  // namespace

int exchange_gather(const ExchangeRanks& ex, const void* src, uint32_t n_local, uint32_t off, void* dst,
                    uint32_t n_total, cudaStream_t stream) {
    if (ex.n_ranks == 0 || ex.n_ranks > kMaxExRanks || ex.rank >= ex.n_ranks)
        return set_error(ARC_E_INVALID_ARGUMENT, "exchange: 1..8 ranks, rank < n_ranks");
    if (!src || !dst || n_total == 0 || n_total > ex.max_words || off + n_local > n_total)
        return set_error(ARC_E_INVALID_ARGUMENT, "exchange: bad slice or vector size");
    return exchange_launch(ex, src, n_local, off, dst, n_total, nullptr, false, stream);
}

int exchange_reduce(const ExchangeRanks& ex, const float* src, uint32_t n, const float* residual, float* dst,
                    cudaStream_t stream) {
    if (ex.n_ranks == 0 || ex.n_ranks > kMaxExRanks || ex.rank >= ex.n_ranks)
        return set_error(ARC_E_INVALID_ARGUMENT, "exchange: 1..8 ranks, rank < n_ranks");
    if (!src || !dst || n == 0 || (uint64_t)n * ex.n_ranks > ex.max_words)
        return set_error(ARC_E_INVALID_ARGUMENT, "exchange reduce: n_ranks * n exceeds the buffer");
    if (dst == residual || dst == src) return set_error(ARC_E_INVALID_ARGUMENT, "exchange reduce: dst must not alias");
    return exchange_launch(ex, src, n, ex.rank * n, dst, n, residual, true, stream);
}

// Contiguous shard [row0, row0 + rows) of n rows for `rank` of n_ranks: whole
// units of `align` rows, the remainder units going one each to the first ranks.
int shard_rows(uint32_t n, uint32_t align, uint32_t n_ranks, uint32_t rank, uint32_t* row0, uint32_t* rows) {
    if (!row0 || !rows || align == 0 || n_ranks == 0 || rank >= n_ranks || n % align)
        return set_error(ARC_E_INVALID_ARGUMENT, "shard_rows: n must be a multiple of align, rank < n_ranks");
    const uint32_t units = n / align, base = units / n_ranks, extra = units % n_ranks;
    if (base == 0) return set_error(ARC_E_UNSUPPORTED_SHAPE, "shard_rows: fewer units than ranks");
    const uint32_t u0 = rank * base + (rank < extra ? rank : extra);
    *row0 = u0 * align;
    *rows = (base + (rank < extra ? 1u : 0u)) * align;
    return ARC_OK;
}

}  // namespace arc
