// Rank exchange over NVLink peer stores: the all-gather steps of the
// row-sharded decode (tensor-parallel generate()).
//
// The reference decodes on one device (src/arcllm_v1_runtime.cpp:371-421, one
// Vulkan queue, src/arcllm_v1_vulkan_runtime_support.h:535).  Sharded over N
// GPUs, the FFN gate/up rows, the FFN down rows and the LM-head rows are split
// over the ranks, and three vectors must be reassembled on every rank: s
// (the SiLU*up product, 18944 floats at the Qwen2.5-7B shape), the new hidden
// state h (3584 floats) and the greedy-selection records (4 words per rank).
//
// exchange_gather_kernel is one 128-thread CTA per rank.  It stores this rank's slice of
// the vector (or, in the reduce form, its whole partial vector into slot
// `rank`) into every rank's exchange buffer (its own with local stores,
// the others with NVLink peer stores -- stores only, nothing reads another
// GPU's memory), fences at system scope, publishes the exchange's sequence
// number in its slot of every rank's flag array (release) and waits (acquire,
// bounded by %globaltimer) until every slot of its own array has reached it;
// then it copies the assembled vector out of its own buffer into `dst` (reduce
// form: adds the ranks' slots in rank order, plus an optional residual -- the
// all-reduce of the K-sharded FFN down projection).
//
// Buffer of one rank (32-bit words; W = the largest vector rounded up to 4):
//   [0, 2W)        two data regions, picked by the parity of the sequence number
//   [2W, 2W+8)     flag array: slot r holds the last sequence number rank r published
//   [2W+8]         this rank's sequence counter (local; advanced by each exchange)
// Every rank runs the same exchanges in the same order (the decode graph), so
// the counters agree without host involvement and a graph replays unchanged.
// Why two regions suffice: a rank can store into a peer's region of sequence
// e+2 only after that peer published e+1, i.e. after its exchange e (which
// reads the same region) completed -- the exchanges of one rank are stream
// ordered.  A wait that runs out sets the device error word's timeout bit and
// returns without the copy; the ranks' counters may then disagree, so the
// exchange buffers must be re-created (zeroed) before further use.
#include "arcllm_cuda_internal.h"
#include "common.cuh"
#include "decode_ops.h"

namespace arc {
namespace {

constexpr uint32_t kFlagWords = 8;
constexpr uint32_t kMaxExRanks = 8;

struct ExParams {
    uint32_t* data[kMaxExRanks];   // rank q's buffer base (its data regions), as this process maps it
    uint32_t* flags[kMaxExRanks];  // rank q's flag array
    uint32_t* seq;                 // this rank's counter
    const uint32_t* src;           // this rank's slice
    uint32_t* dst;                 // the assembled vector (n_total words)
    uint32_t W, n_local, off, n_total, n_ranks, rank;
    unsigned long long wait_ns;
    unsigned int* err;
    // reduce form: every rank contributes a whole n_total-float vector (slot `rank` of the
    // region) and dst = residual (nullable) + the slots added in rank order
    uint32_t reduce;
    const float* residual;
};

// 128 threads of at most 32 registers: 4096 registers, which fit beside one CTA
// of the matvec kernels (480 threads x <= 128 registers), so the exchange is
// resident -- launched early by programmatic dependent launch, parked in
// griddepcontrol.wait -- when the kernel producing its slice ends.
constexpr uint32_t kExThreads = 128;

__global__ void __launch_bounds__(kExThreads, 16) exchange_gather_kernel(const ExParams p) {
    __shared__ uint32_t s_seq;
    __shared__ int s_ok;
    pdl_trigger();
    pdl_wait();  // the slice comes from the preceding kernel
    const uint32_t tid = threadIdx.x, nt = blockDim.x;
    if (tid == 0) s_seq = *reinterpret_cast<volatile uint32_t*>(p.seq) + 1u;
    __syncthreads();
    const uint32_t seq = s_seq, region = (seq & 1u) * p.W;
    const bool vec = ((p.off | p.n_local) & 3u) == 0u && (reinterpret_cast<uintptr_t>(p.src) & 15u) == 0u;
    for (uint32_t q = 0; q < p.n_ranks; ++q) {
        uint32_t* d = p.data[q] + region + p.off;
        if (vec) {
            const uint4* s4 = reinterpret_cast<const uint4*>(p.src);
            uint4* d4 = reinterpret_cast<uint4*>(d);
            for (uint32_t i = tid; i < p.n_local / 4u; i += nt) d4[i] = s4[i];
        } else {
            for (uint32_t i = tid; i < p.n_local; i += nt) d[i] = p.src[i];
        }
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence_system();  // this CTA's (peer) stores before the flags
        for (uint32_t q = 0; q < p.n_ranks; ++q)
            asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p.flags[q] + p.rank), "r"(seq) : "memory");
        const uint32_t* mine = p.flags[p.rank];
        const unsigned long long t0 = globaltimer();
        int ok = 1;
        for (uint32_t q = 0; q < p.n_ranks && ok; ++q) {
            for (;;) {
                uint32_t v;
                asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine + q) : "memory");
                if ((int)(v - seq) >= 0) break;
                if (globaltimer() - t0 > p.wait_ns) {
                    raise_error(p.err, ARC_DEV_ERR_TIMEOUT);
                    ok = 0;
                    break;
                }
                __nanosleep(32);
            }
        }
        *p.seq = seq;
        s_ok = ok;
    }
    __syncthreads();
    if (!s_ok) return;
    // the peers' stores landed in this GPU's memory; read them from L2, not a stale L1 line
    const uint32_t* own = p.data[p.rank] + region;
    if (p.reduce) {  // the same sum, in the same order, on every rank
        const float* slots = reinterpret_cast<const float*>(own);
        float* out = reinterpret_cast<float*>(p.dst);
        for (uint32_t i = tid; i < p.n_total; i += nt) {
            float t = __ldcg(slots + i);
            for (uint32_t q = 1; q < p.n_ranks; ++q) t += __ldcg(slots + (uint64_t)q * p.n_total + i);
            out[i] = p.residual ? p.residual[i] + t : t;
        }
        return;
    }
    if ((p.n_total & 3u) == 0u && (reinterpret_cast<uintptr_t>(p.dst) & 15u) == 0u) {
        const uint4* s4 = reinterpret_cast<const uint4*>(own);
        uint4* d4 = reinterpret_cast<uint4*>(p.dst);
        for (uint32_t i = tid; i < p.n_total / 4u; i += nt) d4[i] = __ldcg(s4 + i);
    } else {
        for (uint32_t i = tid; i < p.n_total; i += nt) p.dst[i] = __ldcg(own + i);
    }
}

// Data regions are whole 16-byte units, so every region starts 16-byte aligned.
inline uint32_t region_words(uint32_t max_words) { return (max_words + 3u) & ~3u; }

}  // namespace

uint64_t exchange_buffer_bytes(uint32_t max_words) {
    return ((uint64_t)(2u * region_words(max_words) + kFlagWords + 8u) * 4u + 255u) / 256u * 256u;
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
        p.data[q] = static_cast<uint32_t*>(ex.bufs[q]);
        p.flags[q] = p.data[q] + 2u * region_words(ex.max_words);
    }
    p.seq = p.flags[ex.rank] + kFlagWords;
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
    return launch_checked(launch_kernel(exchange_gather_kernel, dim3(1), dim3(kExThreads), 0, stream, p),
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
