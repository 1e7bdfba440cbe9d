// arcllm_cuda_attention_decode_noalloc: the split-KV decode attention with its
// scratch held inside the library instead of supplied by the caller.
//
// Who needs this: some callers cannot allocate device memory when they run a
// decode step.  A host that plans every byte of device memory up front and
// refuses anything outside that plan (ArcLLM's own runtime checks its
// buffers against a fixed residency envelope before it runs anything) has no
// place to put a per-call scratch buffer; a latency-critical loop cannot
// afford cudaMalloc, which may synchronise the whole device; and a plugin
// whose host owns the memory budget may simply not be allowed to allocate.
// For them the partial results of the position slices live in a fixed
// array that is part of this library's device image, so the call takes no
// scratch pointer and allocates nothing.
//
// Limits and behaviour:
//   * the array holds kMaxScratchFloats (65536) floats = 256 KiB, and every
//     GPU that loads the library keeps it until the process exits;
//   * a call needs kv_heads * n_splits * (q_heads / kv_heads) * (head_dim + 2)
//     floats (58,240 for Qwen2.5-7B with 16 splits); larger requests are
//     rejected with ARC_E_UNSUPPORTED_SHAPE and nothing is launched;
//   * the array carries the partials only when the slices are merged by the
//     separate merge kernel (n_splits == 1 or > 16, no schedulable 16-CTA
//     cluster, or ARCLLM_ATTN_CLUSTER=0); the clustered form merges through
//     distributed shared memory and leaves the array untouched.  The size
//     limit is checked either way, as part of the contract;
//   * all calls on a device share the one array: calls whose kernels overlap on
//     the GPU (different streams without ordering) race and corrupt each
//     other's results.  Calls ordered on one stream are safe;
//   * the array keeps the previous call's contents.  Nothing needs clearing:
//     every slot a call reads is written by that same call first;
//   * the first call on each device resolves the array's device address with
//     cudaGetSymbolAddress, so make that first call outside stream capture.
#include <cmath>
#include <mutex>

#include "arcllm_cuda_internal.h"
#include "decode_ops.h"

namespace arc {
namespace {

constexpr uint32_t kMaxScratchFloats = 65536;

static __device__ __align__(256) float g_attention_scratch[kMaxScratchFloats];

std::mutex g_scratch_mutex;
float* g_scratch_ptr[64] = {};

// Device address of g_attention_scratch on the current device (resolved once
// per device; in host code the symbol itself is only a host-side stand-in).
int scratch_for_current_device(float** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_cuda_error(e, "attention_decode_noalloc: cudaGetDevice");
    if (dev < 0 || dev >= 64) return set_error(ARC_E_INVALID_ARGUMENT, "attention_decode_noalloc: device index >= 64");
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_attention_scratch);
        if (e != cudaSuccess || !p) return set_cuda_error(e, "attention_decode_noalloc: cudaGetSymbolAddress");
        g_scratch_ptr[dev] = static_cast<float*>(p);
    }
    *out = g_scratch_ptr[dev];
    return ARC_OK;
}

}  // namespace
}  // namespace arc

extern "C" int arcllm_cuda_attention_decode_noalloc(const float* q, const uint16_t* k_cache, const uint16_t* v_cache,
                                                    const uint32_t* pos_dev, uint32_t q_heads, uint32_t kv_heads,
                                                    uint32_t head_dim, uint32_t max_ctx, uint32_t layer,
                                                    uint32_t n_splits, float* out, void* stream) {
    try {
        if (!q || !k_cache || !v_cache || !pos_dev || !out)
            return arc::set_error(ARC_E_INVALID_ARGUMENT, "attention_decode_noalloc: null pointer");
        if (n_splits == 0 || n_splits > 65535u || kv_heads == 0 || q_heads == 0 || max_ctx == 0 ||
            q_heads % kv_heads)
            return arc::set_error(ARC_E_INVALID_ARGUMENT, "attention_decode_noalloc: bad shape");
        const uint64_t need = (uint64_t)kv_heads * n_splits * (q_heads / kv_heads) * ((uint64_t)head_dim + 2u);
        if (need > arc::kMaxScratchFloats)
            return arc::set_error(ARC_E_UNSUPPORTED_SHAPE,
                                  "attention_decode_noalloc: kv_heads*n_splits*(q_heads/kv_heads)*(head_dim+2) "
                                  "exceeds the fixed 65536-float scratch; use fewer splits or "
                                  "arcllm_cuda_attention_decode with caller scratch");
        float* scratch = nullptr;
        int st = arc::scratch_for_current_device(&scratch);
        if (st != ARC_OK) return st;
        arc::AttnShape s{q_heads, kv_heads, head_dim, max_ctx, layer, n_splits, 1.0f / std::sqrt((float)head_dim)};
        return arc::launch_attention(q, k_cache, v_cache, pos_dev, s, scratch, out, static_cast<cudaStream_t>(stream));
    } catch (...) {
        return arc::set_error(ARC_E_INVALID_ARGUMENT, "attention_decode_noalloc: unexpected C++ exception");
    }
}
