// Shared device helpers for the ArcLLM-B200 kernels (sm_100a only).
//
// * mbarrier + cp.async.bulk (TMA bulk copy) wrappers used by the streaming
//   matvec pipelines;
// * bounded waits: every spin in these kernels gives up after
//   kWaitLimitNs nanoseconds of %globaltimer, records ARC_DEV_ERR_TIMEOUT in
//   the device error word and lets the kernel return, so a lost copy can
//   never wedge the GPU;
// * the fp16 decode used by the bit-exact dequant paths.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "arcllm_b200 kernels are written for sm_100a (B200) only"
#endif

namespace arc {

// device error word bits (read and cleared by arcllm_cuda_device_error)
enum : uint32_t {
    ARC_DEV_ERR_TIMEOUT = 1u,      // a bounded mbarrier / flag wait gave up
    ARC_DEV_ERR_BOUNDS = 2u,       // a kernel rejected an out-of-range index
    ARC_DEV_ERR_RANGE = 4u,        // a value rounded to fp16 left the fp16 range
};

constexpr unsigned long long kWaitLimitNs = 1000000000ull;  // 1 s

__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// `err` is the device error word (arcllm_cuda_device_error reads it); kernels
// receive its address as a parameter.
__device__ __forceinline__ void raise_error(unsigned int* err, uint32_t bits) {
    if (err) atomicOr(err, bits);
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// base + off rounded up to an A-byte boundary of the shared window.  The result
// is derived from base (a pointer into a __shared__ array) by adding an offset,
// so the compiler still knows it addresses shared memory; rounding the pointer
// through an integer would turn every access through it into a generic one
// (measured: the Q6_K LM-head matvec 91.9 -> 77.9 us).
template <uint32_t A>
__device__ __forceinline__ uint8_t* smem_align_up(uint8_t* base, uint32_t off) {
    const uint32_t s = smem_addr(base);
    return base + (((s + off + (A - 1u)) & ~(A - 1u)) - s);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for phase `parity` of `bar` to complete; false (and the device error
// word set) if it did not within kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer() - t0 > kWaitLimitNs) {
            raise_error(err, ARC_DEV_ERR_TIMEOUT);
            return false;
        }
    }
    return true;
}

// L2 policy for weight streams: every weight byte is read once per token, so
// let it leave L2 first and keep activations / KV resident.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// 1-D TMA bulk copy global -> this CTA's shared memory, completing `bytes`
// transactions on `bar`.  dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// 16-byte cp.async global -> shared (L2 only, evict-first hint); src_bytes < 16
// zero-fills the rest of the 16 bytes without reading past src + src_bytes.
// dst and src must be 16-byte aligned.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint32_t src_bytes, uint64_t policy) {
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2, %3;" ::"r"(smem_addr(dst)), "l"(src),
                 "r"(src_bytes), "l"(policy)
                 : "memory");
}

// One arrival on `bar` once every cp.async this thread issued so far has landed
// (the barrier's expected count includes it).
__device__ __forceinline__ void cp_async_mbar_arrive(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// Bit-level fp16 -> fp32 (normal, subnormal, inf and NaN payload preserved),
// so dequantised values match the reference's half_to_float bit for bit.
// Programmatic dependent launch: pdl_wait() blocks until the grids this one
// depends on have completed and their writes are visible (a no-op for a
// launch without a programmatic dependency); pdl_trigger() lets the dependent
// grid be scheduled once every CTA of this grid has triggered or exited.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ float half_bits_to_float(uint32_t h) {
    const uint32_t sign = (h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t mant = h & 0x3ffu;
    uint32_t out;
    if (exp == 0u) {
        if (mant == 0u) {
            out = sign;
        } else {
            // subnormal: normalise (the leading one is at bit 9 - (clz - 22))
            const int lz = __clz(mant) - 21;  // shifts to bring bit 10 set
            mant = (mant << lz) & 0x3ffu;
            out = sign | (uint32_t(127 - 14 - lz) << 23) | (mant << 13);
        }
    } else if (exp == 31u) {
        out = sign | 0x7f800000u | (mant << 13);
    } else {
        out = sign | ((exp + 112u) << 23) | (mant << 13);
    }
    return __uint_as_float(out);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Relaxed GPU-scope 64-bit accesses, for tagged words exchanged between CTAs of one device.
__device__ __forceinline__ void st_relaxed_gpu_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_gpu_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Relaxed system-scope 64-bit accesses: single-copy atomic, so a word that
// carries its own epoch tag next to its value needs no fence on either side.
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Cross-rank flag handshake, run by all 32 lanes of one warp after the stores
// it publishes (this CTA's, ordered before it by a CTA barrier, or other CTAs',
// ordered by a counter they incremented after their own fences):
//  1. one system-scope fence: the release for every flag below (and the
//     acquire of a counter read just before);
//  2. lane q < n stores `seq` into slot `self` of rank q's flag array --
//     relaxed system-scope stores, so the n NVLink stores are in flight
//     together instead of each waiting on a fence of its own;
//  3. lane q polls slot q of this rank's own array (relaxed, system scope)
//     until it reaches `seq` (wrap-safe: a peer may already be one ahead);
//  4. one system-scope fence: the acquire, after which the peers' stores
//     that preceded their flags are visible.
// flags[q] is rank q's flag array as this process maps it (n <= NMAX <= 32).
// Gives up after wait_ns, raising ARC_DEV_ERR_TIMEOUT, and returns false.
template <uint32_t NMAX>
__device__ __forceinline__ bool rank_flag_handshake(uint32_t* const (&flags)[NMAX], uint32_t n, uint32_t self,
                                                    uint32_t seq, unsigned long long wait_ns, unsigned int* err) {
    static_assert(NMAX <= 32, "one lane per rank");
    const uint32_t lane = threadIdx.x & 31u;
    uint32_t* peer = nullptr;
    const uint32_t* mine = nullptr;
#pragma unroll
    for (uint32_t q = 0; q < NMAX; ++q) {  // constant indices: the parameter array stays in param space
        if (q == lane) peer = flags[q];
        if (q == self) mine = flags[q];
    }
    __threadfence_system();
    if (lane < n) asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(peer + self), "r"(seq) : "memory");
    const unsigned long long t0 = globaltimer();
    bool seen = lane >= n;
    for (;;) {
        if (!seen) {
            uint32_t v;
            asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine + lane) : "memory");
            seen = (int)(v - seq) >= 0;
        }
        if (__all_sync(0xffffffffu, seen)) break;
        if (__shfl_sync(0xffffffffu, (globaltimer() - t0 > wait_ns) ? 1 : 0, 0)) {
            if (lane == 0) raise_error(err, ARC_DEV_ERR_TIMEOUT);
            return false;
        }
        __nanosleep(32);
    }
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    return true;
}

}  // namespace arc
