// Decode-step kernels other than the matvecs (B200, sm_100a).
//
//   embed_rows        token embedding gather (fp16 rows -> fp32), the config-3
//                     form of shaders/p8c_embedding_q4k_segmented_probe.comp
//                     (src/arcllm_v1_runtime.cpp:373); Q4_K rows reuse the
//                     bit-exact dequant.
//   rope_kv_store     RoPE on q and k (adjacent pairs (2p, 2p+1), angle
//                     pos*theta^(-2p/d), shaders/p7_rope_seq.comp:15-38) fused
//                     with the KV-cache store (shaders/p7_kv_store.comp:14-25)
//                     into an fp16 cache [layer][ctx][kv_dim].  cos/sin come
//                     from a table the host fills with the reference's own
//                     float expression, so the rotation is bit-exact.
//   attn_partial /    cached GQA decode attention
//   attn_merge        (shaders/p7_attention_kv_online.comp, CPU form
//                     src/p8c_segmented_access_correctness.cpp:1136-1158) as
//                     split-KV: each CTA takes one KV head and a slice of the
//                     positions for all q heads of that group, keeps an online
//                     softmax, and a merge pass combines the slices.  With
//                     at most 16 slices the slices of one KV head form a
//                     thread-block cluster and merge through distributed
//                     shared memory inside the same kernel (same arithmetic
//                     and order as the separate merge kernel, one launch less
//                     per layer).
//   argmax_key /      greedy select (src/arcllm_v1_runtime.cpp:132-148):
//   greedy_finalize   first index of the maximum over finite logits, as a
//                     packed 64-bit key reduced with atomicMax; a one-thread
//                     kernel turns it into the next token on the device.
#include <atomic>
#include <cfloat>
#include <cstdlib>
#include <mutex>

#include <cooperative_groups.h>

#include "arcllm_cuda_internal.h"
#include "common.cuh"
#include "decode_ops.h"

namespace arc {
namespace {

__global__ void embed_f16_kernel(const uint16_t* __restrict__ table, const uint32_t* __restrict__ token_src,
                                 uint32_t h, uint32_t vocab, float* __restrict__ out, unsigned int* err) {
    pdl_trigger();
    pdl_wait();  // inputs come from the preceding kernels
    const uint32_t tok = token_src[blockIdx.z];  // row z of a batch (one row for a decode step)
    out += (uint64_t)blockIdx.z * h;
    if (tok >= vocab) {
        if (threadIdx.x == 0 && blockIdx.x == 0) raise_error(err, ARC_DEV_ERR_BOUNDS);
        return;
    }
    const uint16_t* row = table + (uint64_t)tok * h;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < h; i += gridDim.x * blockDim.x)
        out[i] = half_bits_to_float(row[i]);
}

__global__ void embed_q4k_kernel(const uint8_t* __restrict__ table, const uint32_t* __restrict__ token_src,
                                 uint32_t h, uint32_t vocab, float* __restrict__ out, unsigned int* err) {
    pdl_trigger();
    pdl_wait();  // inputs come from the preceding kernels
    const uint32_t tok = token_src[blockIdx.z];  // row z of a batch (one row for a decode step)
    out += (uint64_t)blockIdx.z * h;
    if (tok >= vocab) {
        if (threadIdx.x == 0 && blockIdx.x == 0) raise_error(err, ARC_DEV_ERR_BOUNDS);
        return;
    }
    const uint32_t nb = h / 256u;
    const uint32_t ib = blockIdx.x;  // one super-block per CTA, 256 threads
    if (ib >= nb) return;
    const uint8_t* b = table + ((uint64_t)tok * nb + ib) * 144u;
    const uint32_t k = threadIdx.x;
    const float d = half_bits_to_float((uint32_t)b[0] | ((uint32_t)b[1] << 8));
    const float dmin = half_bits_to_float((uint32_t)b[2] | ((uint32_t)b[3] << 8));
    const uint8_t* q = b + 4;
    const uint32_t j = k >> 5;
    uint32_t sc, mn;
    if (j < 4) {
        sc = q[j] & 63u;
        mn = q[j + 4] & 63u;
    } else {
        sc = (q[j + 4] & 0xFu) | ((q[j - 4] >> 6) << 4);
        mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
    const uint32_t g = k >> 6, l = k & 63u;
    const uint8_t qb = b[16u + g * 32u + (l & 31u)];
    const uint32_t qv = l < 32u ? (qb & 15u) : (qb >> 4);
    out[ib * 256u + k] = __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)qv), __fmul_rn(dmin, (float)mn));
}

// One thread per rotation pair.  q pairs first, then k pairs; k and v are
// written to the fp16 cache at position *pos_src of `layer`.
__global__ void rope_kv_store_kernel(float* __restrict__ q, float* __restrict__ k, const float* __restrict__ v,
                                     const float2* __restrict__ table, const uint32_t* __restrict__ pos_src,
                                     uint16_t* __restrict__ kc, uint16_t* __restrict__ vc, RopeKvShape s,
                                     unsigned int* err) {
    pdl_trigger();
    pdl_wait();  // inputs come from the preceding kernels
    const uint32_t pos = *pos_src;
    if (pos >= s.max_ctx) {
        if (threadIdx.x == 0 && blockIdx.x == 0) raise_error(err, ARC_DEV_ERR_BOUNDS);
        return;
    }
    const uint32_t half = s.head_dim / 2u;
    const uint32_t nq = s.q_heads * half, nk = s.kv_heads * half;
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    const float2* tr = table + (uint64_t)pos * half;
    const uint32_t kv_dim = s.kv_heads * s.head_dim;
    const uint64_t cbase = ((uint64_t)s.layer * s.max_ctx + pos) * kv_dim;
    if (i < nq) {
        const uint32_t hh = i / half, pp = i - hh * half;
        const float2 cs = tr[pp];
        float* x = q + hh * s.head_dim + 2u * pp;
        const float a = x[0], b = x[1];
        x[0] = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
        x[1] = __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x));
    } else if (i < nq + nk) {
        const uint32_t j = i - nq, hh = j / half, pp = j - hh * half;
        const float2 cs = tr[pp];
        const uint32_t o = hh * s.head_dim + 2u * pp;
        const float a = k[o], b = k[o + 1];
        const float r0 = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
        const float r1 = __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x));
        k[o] = r0;
        k[o + 1] = r1;
        kc[cbase + o] = __half_as_ushort(__float2half_rn(r0));
        kc[cbase + o + 1] = __half_as_ushort(__float2half_rn(r1));
        vc[cbase + o] = __half_as_ushort(__float2half_rn(v[o]));
        vc[cbase + o + 1] = __half_as_ushort(__float2half_rn(v[o + 1]));
    }
}

// Slices actually holding positions when n positions are split n_splits ways.
__device__ __forceinline__ uint32_t attn_used_slices(uint32_t n, uint32_t n_splits) {
    const uint32_t chunk = (n + n_splits - 1u) / n_splits;
    return (n + chunk - 1u) / chunk;
}

// Merge the `used` slices of one output (q head, dim): an online merge over
// chunks of 8 slices whose (max, sum, acc) loads are all issued before any is
// used.  slice(sp, m, l, a) loads slice sp's values.
template <typename Slice>
__device__ __forceinline__ float attn_merge_slices(uint32_t used, Slice slice) {
    constexpr int CH = 8;
    float M = -FLT_MAX, L = 0.f, A = 0.f;
    for (uint32_t sp0 = 0; sp0 < used; sp0 += CH) {
        float mm[CH], ll[CH], aa[CH];
#pragma unroll
        for (int j = 0; j < CH; ++j) {
            const uint32_t sp = sp0 + j;
            if (sp < used) {
                slice(sp, mm[j], ll[j], aa[j]);
            } else {
                mm[j] = -FLT_MAX, ll[j] = 0.f, aa[j] = 0.f;
            }
        }
        float cm = M;
#pragma unroll
        for (int j = 0; j < CH; ++j) cm = fmaxf(cm, mm[j]);
        const float r = __expf(M - cm);
        L *= r;
        A *= r;
#pragma unroll
        for (int j = 0; j < CH; ++j) {
            const float f = __expf(mm[j] - cm);
            L = fmaf(ll[j], f, L);
            A = fmaf(aa[j], f, A);
        }
        M = cm;
    }
    return A / L;
}

// Split-KV attention, one CTA per (slice, kv head).  Warps stride over the
// slice's positions; each lane owns 4 of the 128 head dims, holds all G q
// heads of the group in registers, and keeps an online softmax per head.
// CLUSTER: the kv head's slices are one thread-block cluster (grid.x =
// n_splits <= 16); each CTA leaves its slice result in shared memory, the
// cluster synchronises, and CTA c of C merges outputs 256c + 256C*j + t of the
// kv head from all slices' shared memory, writing `out` directly.  Otherwise the
// slice results go to `part` for attn_merge_kernel.
template <int GQ, bool CLUSTER>
__global__ void __launch_bounds__(256) attn_partial_kernel(const float* __restrict__ q,
                                                           const uint16_t* __restrict__ kc,
                                                           const uint16_t* __restrict__ vc,
                                                           const uint32_t* __restrict__ pos_src, AttnShape s,
                                                           float* __restrict__ part, float* __restrict__ out) {
    pdl_trigger();
    pdl_wait();  // inputs come from the preceding kernels
    constexpr int D = 128, NW = 8;
    __shared__ float sm_m[NW][GQ], sm_l[NW][GQ];
    __shared__ float sm_acc[NW][GQ][D];
    const uint32_t split = blockIdx.x, kvh = blockIdx.y;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t pos = min(*pos_src, s.max_ctx - 1u);
    const uint32_t n = pos + 1u;
    const uint32_t chunk = (n + s.n_splits - 1u) / s.n_splits;
    const uint32_t t0 = split * chunk, t1 = min(n, t0 + chunk);
    const uint32_t kv_dim = s.kv_heads * D;
    float qv[GQ][4];
#pragma unroll
    for (int g = 0; g < GQ; ++g) {
        const float4 t = *reinterpret_cast<const float4*>(q + (kvh * GQ + g) * D + lane * 4u);
        qv[g][0] = t.x * s.scale, qv[g][1] = t.y * s.scale, qv[g][2] = t.z * s.scale, qv[g][3] = t.w * s.scale;
    }
    float m[GQ], l[GQ], acc[GQ][4];
#pragma unroll
    for (int g = 0; g < GQ; ++g) {
        m[g] = -FLT_MAX, l[g] = 0.f;
        acc[g][0] = acc[g][1] = acc[g][2] = acc[g][3] = 0.f;
    }
    const uint64_t lbase = (uint64_t)s.layer * s.max_ctx * kv_dim + kvh * D + lane * 4u;
    for (uint32_t t = t0 + warp; t < t1; t += NW) {
        const uint2 kraw = *reinterpret_cast<const uint2*>(kc + lbase + (uint64_t)t * kv_dim);
        const uint2 vraw = *reinterpret_cast<const uint2*>(vc + lbase + (uint64_t)t * kv_dim);
        const float2 k01 = __half22float2(*reinterpret_cast<const __half2*>(&kraw.x));
        const float2 k23 = __half22float2(*reinterpret_cast<const __half2*>(&kraw.y));
        const float2 v01 = __half22float2(*reinterpret_cast<const __half2*>(&vraw.x));
        const float2 v23 = __half22float2(*reinterpret_cast<const __half2*>(&vraw.y));
        float sc[GQ];
#pragma unroll
        for (int g = 0; g < GQ; ++g)
            sc[g] = fmaf(qv[g][0], k01.x, fmaf(qv[g][1], k01.y, fmaf(qv[g][2], k23.x, qv[g][3] * k23.y)));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
            for (int g = 0; g < GQ; ++g) sc[g] += __shfl_xor_sync(0xffffffffu, sc[g], o);
        }
#pragma unroll
        for (int g = 0; g < GQ; ++g) {
            const float mn = fmaxf(m[g], sc[g]);
            const float a = __expf(m[g] - mn), p = __expf(sc[g] - mn);
            l[g] = fmaf(l[g], a, p);
            acc[g][0] = fmaf(acc[g][0], a, p * v01.x);
            acc[g][1] = fmaf(acc[g][1], a, p * v01.y);
            acc[g][2] = fmaf(acc[g][2], a, p * v23.x);
            acc[g][3] = fmaf(acc[g][3], a, p * v23.y);
            m[g] = mn;
        }
    }
#pragma unroll
    for (int g = 0; g < GQ; ++g) {
        if (lane == 0) sm_m[warp][g] = m[g], sm_l[warp][g] = l[g];
        *reinterpret_cast<float4*>(&sm_acc[warp][g][lane * 4u]) = make_float4(acc[g][0], acc[g][1], acc[g][2], acc[g][3]);
    }
    __syncthreads();
    __shared__ float res[CLUSTER ? GQ : 1][D + 2];  // this slice's (max, sum, acc[128]) per q head
    // combine the 8 warps: thread (g, d) for g < GQ, d < 128 (GQ*128 <= 1024, two passes of 256 threads... )
    for (uint32_t idx = threadIdx.x; idx < GQ * D; idx += 256u) {
        const uint32_t g = idx / D, d = idx - g * D;
        float M = -FLT_MAX;
#pragma unroll
        for (int w = 0; w < NW; ++w) M = fmaxf(M, sm_m[w][g]);
        float L = 0.f, A = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            const float f = __expf(sm_m[w][g] - M);
            L = fmaf(sm_l[w][g], f, L);
            A = fmaf(sm_acc[w][g][d], f, A);
        }
        float* o = CLUSTER ? &res[g][0] : part + (((uint64_t)kvh * s.n_splits + split) * GQ + g) * (D + 2u);
        o[2 + d] = A;
        if (d == 0) o[0] = M, o[1] = L;
    }
    if constexpr (CLUSTER) {
        namespace cg = cooperative_groups;
        cg::cluster_group cl = cg::this_cluster();
        cl.sync();  // every slice's result is in its CTA's shared memory
        const uint32_t used = attn_used_slices(n, s.n_splits);
        for (uint32_t o = cl.block_rank() * 256u + threadIdx.x; o < GQ * D; o += cl.num_blocks() * 256u) {
            const uint32_t g = o / D, d = o - g * D;
            out[(kvh * GQ + g) * D + d] = attn_merge_slices(used, [&](uint32_t sp, float& mm, float& ll, float& aa) {
                const float* r = cl.map_shared_rank(&res[g][0], sp);
                mm = r[0], ll = r[1], aa = r[2 + d];
            });
        }
        cl.sync();  // no CTA leaves while the others still read its shared memory
    }
}

// Merge the slices of one q head (the form without a cluster).
__global__ void attn_merge_kernel(const float* __restrict__ part, const uint32_t* __restrict__ pos_src, AttnShape s,
                                  uint32_t gq, float* __restrict__ out) {
    pdl_trigger();
    pdl_wait();  // inputs come from the preceding kernels
    constexpr int D = 128;
    const uint32_t qh = blockIdx.x, d = threadIdx.x;
    const uint32_t kvh = qh / gq, g = qh - kvh * gq;
    const uint32_t n = min(*pos_src, s.max_ctx - 1u) + 1u;
    out[qh * D + d] = attn_merge_slices(attn_used_slices(n, s.n_splits), [&](uint32_t sp, float& mm, float& ll,
                                                                            float& aa) {
        const float* pp = part + (((uint64_t)kvh * s.n_splits + sp) * gq + g) * (D + 2u);
        mm = pp[0], ll = pp[1], aa = pp[2 + d];
    });
}

// orderable encoding of a float: larger float -> larger unsigned; -0.0 and
// +0.0 compare equal (as with the reference's float '>'), so both map to +0.
__device__ __forceinline__ uint32_t f2ord(float f) {
    uint32_t u = __float_as_uint(f);
    if (u == 0x80000000u) u = 0u;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// key = ord(value) << 32 | ~index : atomicMax keeps the largest value and,
// among equal values, the smallest index (the reference's strict '>' scan).
__global__ void argmax_key_kernel(const float* __restrict__ logits, uint32_t n, uint32_t base,
                                  unsigned long long* key_out, uint32_t* nonfinite_out) {
    pdl_trigger();
    pdl_wait();  // inputs come from the preceding kernels
    unsigned long long best = 0ull;
    uint32_t nonfinite = 0;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float v = logits[i];
        if (!isfinite(v)) {
            nonfinite = 1u;
            continue;
        }
        const unsigned long long key = ((unsigned long long)f2ord(v) << 32) | (unsigned long long)(~(base + i));
        best = key > best ? key : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
        nonfinite |= __shfl_xor_sync(0xffffffffu, nonfinite, o);
    }
    if ((threadIdx.x & 31u) == 0) {
        if (best) atomicMax(key_out, best);
        if (nonfinite) atomicOr(nonfinite_out, 1u);
    }
}

// Tensor-parallel greedy select: the ranks' (nonfinite, pad, key lo, key hi)
// records, gathered in rank order, combined into this rank's state -- the
// largest key (the first index of the maximum over all shards, since each
// key carries the complemented global index) and any non-finite flag.
__global__ void greedy_combine_kernel(GreedyState* st, const uint32_t* __restrict__ recs, uint32_t n_ranks) {
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    unsigned long long best = 0ull;
    uint32_t nonfinite = 0;
    for (uint32_t q = 0; q < n_ranks; ++q) {
        nonfinite |= recs[4u * q];
        const unsigned long long key = (unsigned long long)recs[4u * q + 2u] |
                                       ((unsigned long long)recs[4u * q + 3u] << 32);
        best = key > best ? key : best;
    }
    st->argmax_key = best;
    st->nonfinite |= nonfinite;
}

// Advance the decode state by one token: next token = prompt[pos+1] while the
// prompt is being consumed, else the greedy argmax; record generated tokens.
__global__ void greedy_finalize_kernel(GreedyState* st, const uint32_t* __restrict__ prompt, uint32_t* out_tokens,
                                       uint32_t max_out) {
    pdl_trigger();
    pdl_wait();  // inputs come from the preceding kernels
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    const uint32_t pos = st->pos;
    uint32_t next;
    if (pos + 1u < st->n_prompt) {
        next = prompt[pos + 1u];
    } else {
        const unsigned long long key = st->argmax_key;
        next = key ? ~(uint32_t)(key & 0xffffffffull) : 0u;
        if (!key) st->nonfinite |= 2u;
        if (st->n_generated < max_out) out_tokens[st->n_generated] = next;
        st->n_generated += 1u;
    }
    st->argmax_key = 0ull;
    st->token = next;
    st->pos = pos + 1u;
}

}  // namespace

int decode_ops_prepare() {
    cudaFuncAttributes a;
    cudaError_t e = cudaFuncGetAttributes(&a, embed_f16_kernel);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&a, embed_q4k_kernel);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&a, rope_kv_store_kernel);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&a, attn_partial_kernel<1, false>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&a, attn_partial_kernel<2, false>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&a, attn_partial_kernel<4, false>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&a, attn_partial_kernel<7, false>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&a, attn_partial_kernel<8, false>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&a, attn_merge_kernel);
    // clusters of up to 16 slices (16 is beyond the portable 8: opt in per kernel)
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attn_partial_kernel<1, true>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attn_partial_kernel<2, true>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attn_partial_kernel<4, true>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attn_partial_kernel<7, true>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attn_partial_kernel<8, true>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&a, argmax_key_kernel);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&a, greedy_finalize_kernel);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&a, greedy_combine_kernel);
    return e == cudaSuccess ? ARC_OK : set_cuda_error(e, "decode ops prepare");
}

int launch_checked(cudaError_t e, const char* what) { return e == cudaSuccess ? ARC_OK : set_cuda_error(e, what); }

int launch_embed(int type, const void* table, const uint32_t* token_src, uint32_t h, uint32_t vocab, float* out,
                 cudaStream_t stream) {
    return launch_embed_rows(type, table, token_src, 1, h, vocab, out, stream);
}

int launch_embed_rows(int type, const void* table, const uint32_t* token_src, uint32_t rows, uint32_t h,
                      uint32_t vocab, float* out, cudaStream_t stream) {
    if (rows == 0 || rows > 65535u) return set_error(ARC_E_INVALID_ARGUMENT, "embedding: 1..65535 rows");
    if (type == 1)
        return launch_checked(launch_kernel(embed_f16_kernel, dim3((h + 255) / 256, 1, rows), dim3(256), 0, stream,
                                            static_cast<const uint16_t*>(table), token_src, h, vocab, out,
                                            dev_error_word()),
                              "embed launch");
    if (type == 12)
        return launch_checked(launch_kernel(embed_q4k_kernel, dim3(h / 256, 1, rows), dim3(256), 0, stream,
                                            static_cast<const uint8_t*>(table), token_src, h, vocab, out,
                                            dev_error_word()),
                              "embed launch");
    return set_error(ARC_E_UNSUPPORTED_SHAPE, "embedding: type must be F16 (1) or Q4_K (12)");
}

int launch_rope_kv_store(float* q, float* k, const float* v, const float2* table, const uint32_t* pos_src,
                         uint16_t* kc, uint16_t* vc, const RopeKvShape& s, cudaStream_t stream) {
    const uint32_t pairs = (s.q_heads + s.kv_heads) * (s.head_dim / 2u);
    return launch_checked(launch_kernel(rope_kv_store_kernel, dim3((pairs + 127) / 128), dim3(128), 0, stream, q, k, v,
                                        table, pos_src, kc, vc, s, dev_error_word()),
                          "rope_kv_store launch");
}

namespace {

// The cluster form: one launch, grid (n_splits, kv_heads), clusters of n_splits CTAs.
template <int GQ>
cudaError_t launch_attn_cluster(dim3 grid, cudaStream_t stream, const float* q, const uint16_t* kc,
                                const uint16_t* vc, const uint32_t* pos_src, const AttnShape& s, float* out) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = grid.x;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (pdl_enabled()) {
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        cfg.numAttrs = 2;
    }
    const cudaError_t e = cudaLaunchKernelEx(&cfg, attn_partial_kernel<GQ, true>, q, kc, vc, pos_src, s,
                                             static_cast<float*>(nullptr), out);
    return e != cudaSuccess ? e : cudaGetLastError();
}

// Whether clusters of `size` CTAs of the GQ cluster kernel fit on this device (asked once per
// device and size under a lock, so host threads making their first call together agree;
// devices 64 and up take the two-kernel form; ARCLLM_ATTN_CLUSTER=0 turns the cluster form off).
template <int GQ>
bool attn_cluster_ok(uint32_t size, uint32_t kv_heads) {
    static std::atomic<int> known[64][17] = {};  // 0 unknown, 1 yes, 2 no
    static std::mutex probe_mutex;
    if (size < 2u || size > 16u || kv_heads == 0u) return false;
    if (const char* v = std::getenv("ARCLLM_ATTN_CLUSTER"))
        if (v[0] == '0') return false;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    if (dev < 0 || dev >= 64) return false;
    std::atomic<int>& k = known[dev][size];
    if (k.load(std::memory_order_acquire) == 0) {
        std::lock_guard<std::mutex> lock(probe_mutex);
        if (k.load(std::memory_order_relaxed) != 0) return k.load(std::memory_order_relaxed) == 1;
        // callers of the C ABI may not have run decode_ops_prepare: opt in to 16-CTA clusters here too
        if (size > 8u &&
            cudaFuncSetAttribute(attn_partial_kernel<GQ, true>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) !=
                cudaSuccess)
            cudaGetLastError();
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(size, kv_heads);
        cfg.blockDim = dim3(256);
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = size;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        const cudaError_t e = cudaOccupancyMaxActiveClusters(&n, attn_partial_kernel<GQ, true>, &cfg);
        if (e != cudaSuccess) cudaGetLastError();
        k.store((e == cudaSuccess && n > 0) ? 1 : 2, std::memory_order_release);
    }
    return k.load(std::memory_order_acquire) == 1;
}

template <int GQ>
cudaError_t launch_attn_gq(dim3 grid, cudaStream_t stream, const float* q, const uint16_t* kc, const uint16_t* vc,
                           const uint32_t* pos_src, const AttnShape& s, float* part, float* out, bool* clustered) {
    *clustered = attn_cluster_ok<GQ>(s.n_splits, s.kv_heads);
    if (*clustered) return launch_attn_cluster<GQ>(grid, stream, q, kc, vc, pos_src, s, out);
    return launch_kernel(attn_partial_kernel<GQ, false>, grid, dim3(256), 0, stream, q, kc, vc, pos_src, s, part, out);
}

}  // namespace

int launch_attention(const float* q, const uint16_t* kc, const uint16_t* vc, const uint32_t* pos_src,
                     const AttnShape& s, float* part, float* out, cudaStream_t stream) {
    if (s.head_dim != 128u) return set_error(ARC_E_UNSUPPORTED_SHAPE, "attention: head_dim must be 128");
    const uint32_t gq = s.q_heads / s.kv_heads;
    if (gq * s.kv_heads != s.q_heads || gq > 8u || gq == 0u)
        return set_error(ARC_E_UNSUPPORTED_SHAPE, "attention: q_heads must be 1..8 x kv_heads");
    dim3 grid(s.n_splits, s.kv_heads);
    cudaError_t e;
    bool clustered = false;
    switch (gq) {
        case 1: e = launch_attn_gq<1>(grid, stream, q, kc, vc, pos_src, s, part, out, &clustered); break;
        case 2: e = launch_attn_gq<2>(grid, stream, q, kc, vc, pos_src, s, part, out, &clustered); break;
        case 4: e = launch_attn_gq<4>(grid, stream, q, kc, vc, pos_src, s, part, out, &clustered); break;
        case 7: e = launch_attn_gq<7>(grid, stream, q, kc, vc, pos_src, s, part, out, &clustered); break;
        case 8: e = launch_attn_gq<8>(grid, stream, q, kc, vc, pos_src, s, part, out, &clustered); break;
        default: return set_error(ARC_E_UNSUPPORTED_SHAPE, "attention: q heads per kv head must be 1, 2, 4, 7 or 8");
    }
    if (e == cudaSuccess && !clustered)
        e = launch_kernel(attn_merge_kernel, dim3(s.q_heads), dim3(128), 0, stream, part, pos_src, s, gq, out);
    return e == cudaSuccess ? ARC_OK : set_cuda_error(e, "attention launch");
}

int attention_launches(uint32_t n_splits, uint32_t q_heads, uint32_t kv_heads) {
    const uint32_t gq = kv_heads ? q_heads / kv_heads : 0u;
    bool c = false;
    switch (gq) {
        case 1: c = attn_cluster_ok<1>(n_splits, kv_heads); break;
        case 2: c = attn_cluster_ok<2>(n_splits, kv_heads); break;
        case 4: c = attn_cluster_ok<4>(n_splits, kv_heads); break;
        case 7: c = attn_cluster_ok<7>(n_splits, kv_heads); break;
        case 8: c = attn_cluster_ok<8>(n_splits, kv_heads); break;
        default: break;
    }
    return c ? 1 : 2;
}

int launch_argmax(const float* logits, uint32_t n, unsigned long long* key, uint32_t* nonfinite,
                  cudaStream_t stream, uint32_t base) {
    return launch_checked(
        launch_kernel(argmax_key_kernel, dim3(148), dim3(256), 0, stream, logits, n, base, key, nonfinite),
        "argmax launch");
}

int launch_greedy_combine(GreedyState* st, const uint32_t* recs, uint32_t n_ranks, cudaStream_t stream) {
    return launch_checked(launch_kernel(greedy_combine_kernel, dim3(1), dim3(32), 0, stream, st, recs, n_ranks),
                          "greedy combine launch");
}

int launch_greedy_finalize(GreedyState* st, const uint32_t* prompt, uint32_t* out_tokens, uint32_t max_out,
                           cudaStream_t stream) {
    return launch_checked(launch_kernel(greedy_finalize_kernel, dim3(1), dim3(32), 0, stream, st, prompt, out_tokens,
                                        max_out),
                          "finalize launch");
}

}  // namespace arc
