// arcllm::v1::runtime::generate() on a B200 (include/arcllm/v1/runtime.h).
//
// Follows the request flow of the reference runtime
// (src/arcllm_v1_runtime.cpp:149-536): validate the request, read the GGUF
// header, map the file and check the TensorStore invariants, check the
// decoder's tensor census and shapes, upload the weights, run prefill and the
// greedy decode loop, release everything before returning.  The Vulkan
// dispatch recording is replaced by the CUDA model of libarcllm_cuda.so (one
// CUDA graph launch per token, next token chosen on the device).
//
// Where the reference pins the frozen Qwen2.5-7B file exactly (339 tensors,
// 19 fixed arena ranges, the 4,677,120,000-byte payload, :41-131,163-172),
// this runtime checks the same structure derived from the file's own metadata
// (block count, widths, head counts), so smaller synthetic Qwen2 models of the
// same architecture run through the same call.  Request limits are the
// reference's: at most 256 prompt tokens, prompt + new tokens within a
// 4096-position KV cache, every token id inside the vocabulary.
#include "arcllm/v1/runtime.h"

#include <cmath>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "arcllm/v1/gguf.h"
#include "arcllm/v1/q4_cuda_backend.h"
#include "arcllm/v1/q4_down_policy.h"
#include "arcllm_cuda.h"

namespace arcllm::v1::runtime {
namespace {

namespace gg = arcllm::v1::gguf;

constexpr std::uint32_t kMaxSeq = 256;   // runtime.cpp:163 MAXSEQ
constexpr std::uint32_t kMaxCtx = 4096;  // runtime.cpp:163 MAXCTX

[[noreturn]] void fail(const std::string& m) { throw std::runtime_error(m); }

void check(int st, const char* what) {
    if (st != ARC_OK)
        fail(std::string("ArcLLM runtime ") + what + " failed: " + arcllm_cuda_status_string(st) + ": " +
             arcllm_cuda_last_error_message());
}

struct DeviceBuffer {
    void* p = nullptr;
    ~DeviceBuffer() { if (p) arcllm_cuda_free(p); }
};
struct ModelHandle {
    arcllm_cuda_model* m = nullptr;
    ~ModelHandle() { if (m) arcllm_cuda_model_destroy(m); }
};
struct StreamHandle {
    void* s = nullptr;
    ~StreamHandle() { if (s) arcllm_cuda_stream_destroy(s); }
};

std::uint32_t meta_u32(const GgufInfo& g, const std::string& key) {
    auto it = g.scalars.find(key);
    if (it == g.scalars.end()) fail("ArcLLM runtime missing metadata: " + key);
    unsigned long v = 0;
    try {
        v = std::stoul(it->second);
    } catch (...) {
        fail("ArcLLM runtime bad metadata value: " + key);
    }
    if (v == 0 || v > 0xFFFFFFFFul) fail("ArcLLM runtime metadata out of range: " + key);
    return std::uint32_t(v);
}

// A tensor of one of `types` with dims {d0} (vector) or {d0, d1} (matrix).
const GgufTensorInfo* require(const GgufInfo& g, const std::string& name, std::initializer_list<std::uint32_t> types,
                              std::uint64_t d0, std::uint64_t d1) {
    const GgufTensorInfo* t = gg::find_tensor(g, name);
    if (!t) fail("ArcLLM runtime missing graph tensor: " + name);
    bool ok = false;
    for (auto ty : types) ok = ok || t->ggml_type == ty;
    if (!ok) fail("ArcLLM runtime unsupported tensor type for " + name + ": " + std::to_string(t->ggml_type));
    const bool vec = d1 == 0;
    if (vec ? !(t->dims.size() == 1 && t->dims[0] == d0)
            : !(t->dims.size() == 2 && t->dims[0] == d0 && t->dims[1] == d1))
        fail("ArcLLM runtime tensor shape mismatch: " + name);
    if (t->offset % 16) fail("ArcLLM runtime tensor not 16-byte aligned: " + name);
    return t;
}

}  // namespace

RunResult generate(const RunRequest& request) {
    if (request.model_path.empty() || request.shader_dir.empty())
        fail("ArcLLM runtime requires model_path and shader_dir");
    if (request.input_token_ids.empty()) fail("ArcLLM runtime requires at least one input token");
    if (request.max_new_tokens == 0u) fail("ArcLLM runtime requires max_new_tokens >= 1");

    GgufInfo g = GgufReader(request.model_path).read();
    gg::TensorStore store;
    const gg::TensorStoreReport ts = store.inspect(request.model_path, g);
    if (!ts.mapped || !ts.all_bounds_valid || !ts.no_overlap || !ts.supported_types_only || !ts.q4_k_direct_access)
        fail("ArcLLM runtime TensorStore invariants failed" + (ts.error.empty() ? std::string() : ": " + ts.error));

    // ---- architecture from metadata (runtime.cpp:163-185 pins these values) ----
    const std::uint32_t L = meta_u32(g, "qwen2.block_count");
    const std::uint32_t H = meta_u32(g, "qwen2.embedding_length");
    const std::uint32_t QH = meta_u32(g, "qwen2.attention.head_count");
    const std::uint32_t KVH = meta_u32(g, "qwen2.attention.head_count_kv");
    const std::uint32_t FFN = meta_u32(g, "qwen2.feed_forward_length");
    if (H % QH || QH % KVH) fail("ArcLLM runtime head geometry mismatch");
    const std::uint32_t HD = H / QH, KV = KVH * HD;
    if (HD % 2) fail("ArcLLM runtime head_dim must be even for RoPE");
    if (g.tensor_count != 12ull * L + 3ull || g.tensors.size() != 12ull * L + 3ull)
        fail("ArcLLM runtime exact tensor census mismatch");
    float eps = 1e-6f;
    if (auto it = g.scalars.find("qwen2.attention.layer_norm_rms_epsilon"); it != g.scalars.end())
        eps = std::stof(it->second);
    float theta = 1000000.0f;
    if (auto it = g.scalars.find("qwen2.rope.freq_base"); it != g.scalars.end()) theta = std::stof(it->second);

    const GgufTensorInfo* emb = gg::find_tensor(g, "token_embd.weight");
    if (!emb || emb->dims.size() != 2) fail("ArcLLM runtime missing graph tensor: token_embd.weight");
    const std::uint64_t VOC64 = emb->dims[1];
    if (VOC64 == 0 || VOC64 > 0xFFFFFFFFull) fail("ArcLLM runtime vocabulary size out of range");
    const std::uint32_t VOC = std::uint32_t(VOC64);
    constexpr std::uint32_t F32 = gg::F32, F16 = gg::F16, Q4 = gg::Q4_K, Q6 = gg::Q6_K;
    require(g, "token_embd.weight", {Q4, F16}, H, VOC);
    const GgufTensorInfo* outw = require(g, "output.weight", {Q6, Q4}, H, VOC);
    require(g, "output_norm.weight", {F32}, H, 0);

    struct LayerTensors {
        const GgufTensorInfo *an, *qw, *kw, *vw, *qb, *kb, *vb, *ow, *fn, *gw, *uw, *dw;
    };
    std::vector<LayerTensors> layers(L);
    for (std::uint32_t l = 0; l < L; ++l) {
        const std::string p = "blk." + std::to_string(l) + ".";
        LayerTensors& z = layers[l];
        z.an = require(g, p + "attn_norm.weight", {F32}, H, 0);
        z.qw = require(g, p + "attn_q.weight", {Q4}, H, H);
        z.kw = require(g, p + "attn_k.weight", {Q4}, H, KV);
        z.vw = require(g, p + "attn_v.weight", {Q4, Q6}, H, KV);
        z.qb = require(g, p + "attn_q.bias", {F32}, H, 0);
        z.kb = require(g, p + "attn_k.bias", {F32}, KV, 0);
        z.vb = require(g, p + "attn_v.bias", {F32}, KV, 0);
        z.ow = require(g, p + "attn_output.weight", {Q4}, H, H);
        z.fn = require(g, p + "ffn_norm.weight", {F32}, H, 0);
        z.gw = require(g, p + "ffn_gate.weight", {Q4}, H, FFN);
        z.uw = require(g, p + "ffn_up.weight", {Q4}, H, FFN);
        z.dw = require(g, p + "ffn_down.weight", {Q4, Q6}, FFN, H);
    }

    // ---- request limits (runtime.cpp:246-252) ----
    if (request.input_token_ids.size() > kMaxSeq)
        fail("ArcLLM runtime prefill token count exceeds current model/runtime limit");
    const std::uint32_t seq = std::uint32_t(request.input_token_ids.size());
    if (std::uint64_t(seq) + std::uint64_t(request.max_new_tokens) - 1ull > kMaxCtx)
        fail("ArcLLM runtime request exceeds KV context limit");
    for (std::uint32_t id : request.input_token_ids)
        if (id >= VOC) fail("ArcLLM runtime input token out of vocabulary");

    int n_dev = 0;
    check(arcllm_cuda_device_count(&n_dev), "device query");
    if (n_dev <= 0) fail("ArcLLM runtime found no CUDA device");

    // ---- weights: the file's tensor payload as one device arena ----
    // Tensor offsets are relative to data_offset and 16-byte aligned (checked
    // per tensor), so device pointers are arena base + offset.
    std::uint64_t payload = 0;
    for (const auto& t : g.tensors) payload = std::max(payload, t.offset + gg::tensor_nbytes(t));
    StreamHandle stream;
    check(arcllm_cuda_stream_create(&stream.s), "stream create");
    DeviceBuffer arena;
    check(arcllm_cuda_malloc(payload + 256, &arena.p), "weight arena allocation");
    check(arcllm_cuda_memcpy_h2d(arena.p, store.mapped_base() + g.data_offset, payload, stream.s), "weight upload");
    auto dev = [&](const GgufTensorInfo* t) -> const void* {
        return static_cast<const std::uint8_t*>(arena.p) + t->offset;
    };
    auto devf = [&](const GgufTensorInfo* t) { return static_cast<const float*>(dev(t)); };

    arcllm_cuda_model_config cfg{L, H, QH, KVH, HD, FFN, VOC, kMaxCtx, eps, theta};
    ModelHandle model;
    check(arcllm_cuda_model_create(&cfg, &model.m), "model create");
    std::vector<cuda::Q4CudaBackend::Source> q4_down;
    for (std::uint32_t l = 0; l < L; ++l) {
        const LayerTensors& z = layers[l];  // decoder tensors (routed through A until the policy says B)
        arcllm_cuda_layer lay{devf(z.an), dev(z.qw), devf(z.qb), int(z.qw->ggml_type), dev(z.kw), devf(z.kb),
                              int(z.kw->ggml_type), dev(z.vw), devf(z.vb), int(z.vw->ggml_type), dev(z.ow),
                              int(z.ow->ggml_type), devf(z.fn), dev(z.gw), dev(z.uw), int(z.gw->ggml_type),
                              dev(z.dw), int(z.dw->ggml_type)};
        check(arcllm_cuda_model_set_layer(model.m, l, &lay), "layer binding");
        if (z.dw->ggml_type == Q4) q4_down.push_back({l, dev(z.dw), store.tensor_data(g, *z.dw)});
    }
    check(arcllm_cuda_model_set_endpoints(model.m, dev(emb), int(emb->ggml_type),
                                          devf(gg::find_tensor(g, "output_norm.weight")), dev(outw),
                                          int(outw->ggml_type)),
          "endpoint binding");

    // ---- Q4 FFN-down primitive: route per decode step from the policy (runtime.cpp:313-339,461-475) ----
    cuda::Q4CudaBackend q4_backend(q4_down, H, FFN, request.sidecar_path);
    binding_v4::PrimitiveHandle route_a{};
    if (q4_backend.resolve_primitive(cuda::kPrimitiveA, route_a) != binding_v4::BackendStatus::OK)
        fail("ArcLLM runtime Q4 binding not ready");
    const bool profile1 = request.evidence_profile == EvidenceProfile::PROFILE_1;
    binding_v4::RepresentationHandle b_handle{};
    auto runtime_state = [&] {
        cuda::Q4DownRuntime rt;
        rt.b_resident = q4_backend.resident();
        rt.b_identity_valid = q4_backend.validated();
        rt.p3_available = q4_backend.p3_available();
        return rt;
    };
    // Apply one decision the way binding_v4::apply_decision does: evict ->
    // release; acquire -> acquire, validate (release on failure); then the
    // route's primitive must resolve.  Returns the routed primitive.
    std::uint32_t acquire_events = 0, evict_events = 0;
    auto apply = [&](const cuda::Q4DownDecision& d) {
        if (d.lifecycle == cuda::Q4DownLifecycle::EVICT && b_handle) {
            if (q4_backend.release(cuda::kPrimitiveB, b_handle) != binding_v4::BackendStatus::OK)
                fail("ArcLLM runtime Q4 binding not ready");
            b_handle = {};
            ++evict_events;
        }
        if (d.lifecycle == cuda::Q4DownLifecycle::ACQUIRE) {
            if (q4_backend.acquire(d.acquisition, cuda::kPrimitiveB, d.requested_residency_bytes, b_handle) !=
                    binding_v4::BackendStatus::OK ||
                !b_handle)
                fail("ArcLLM runtime Q4 binding not ready: " + q4_backend.last_error());
            if (d.require_post_acquisition_identity_validation &&
                q4_backend.validate(b_handle, cuda::kCapability, cuda::kPrimitiveB) != binding_v4::BackendStatus::OK) {
                q4_backend.release(cuda::kPrimitiveB, b_handle);
                b_handle = {};
                fail("ArcLLM runtime Q4 binding not ready: " + q4_backend.last_error());
            }
            ++acquire_events;
        }
        binding_v4::PrimitiveHandle h{};
        if (q4_backend.resolve_primitive(d.route, h) != binding_v4::BackendStatus::OK)
            fail("ArcLLM runtime Q4 binding not ready");
        return d.route;
    };
    // Decode step di decides with future reuse max_new - 1 - di.  With this
    // bundle the route cannot change inside a request (an image acquired at
    // step 0 stays valid and reusable while reuse > 0), so the decisions are
    // taken up front and the model runs the whole request on that route.
    std::uint32_t route_a_steps = 0, route_b_steps = 0;
    registry::PrimitiveId decode_route = cuda::kPrimitiveA;
    if (q4_backend.has_sources()) {
        for (std::uint32_t di = 0; di + 1u < request.max_new_tokens; ++di) {
            const auto d = cuda::decide_q4_down(profile1, request.request_within_validated_domain,
                                                std::uint64_t(request.max_new_tokens - 1u - di), runtime_state(),
                                                q4_backend.exec_family_bytes());
            const registry::PrimitiveId r = apply(d);
            if (di == 0) decode_route = r;
            else if (r != decode_route) fail("ArcLLM runtime Q4 route changed within request");
            (r == cuda::kPrimitiveB ? route_b_steps : route_a_steps)++;
        }
    } else {
        route_a_steps = request.max_new_tokens - 1u;  // no Q4_K down layer: every step is plain A
    }
    if (decode_route == cuda::kPrimitiveB) {  // rebind the Q4_K down layers to the EXEC148 image
        for (const auto& src : q4_down) {
            const LayerTensors& z = layers[src.layer];
            arcllm_cuda_layer lay{devf(z.an), dev(z.qw), devf(z.qb), int(z.qw->ggml_type), dev(z.kw), devf(z.kb),
                                  int(z.kw->ggml_type), dev(z.vw), devf(z.vb), int(z.vw->ggml_type), dev(z.ow),
                                  int(z.ow->ggml_type), devf(z.fn), dev(z.gw), dev(z.uw), int(z.gw->ggml_type),
                                  q4_backend.exec_image(src.layer), ARC_TYPE_EXEC148};
            check(arcllm_cuda_model_set_layer(model.m, src.layer, &lay), "route B binding");
            // the batched prefill GEMMs keep reading the GGUF Q4_K packing of this layer
            check(arcllm_cuda_model_set_prefill_down(model.m, src.layer, dev(z.dw), int(z.dw->ggml_type)),
                  "route B prefill binding");
        }
    }

    // ---- prefill + greedy decode ----
    RunResult result;
    result.generated_token_ids.assign(request.max_new_tokens, 0u);
    arcllm_cuda_gen_stats st{};
    const int rc = arcllm_cuda_model_generate(model.m, request.input_token_ids.data(), seq, request.max_new_tokens,
                                              result.generated_token_ids.data(), &st, stream.s);
    if (rc == ARC_E_NONFINITE) fail("ArcLLM runtime non-finite logits");
    check(rc, "generate");
    if (!st.finite) fail("ArcLLM runtime non-finite logits");
    if (st.decode_steps + 1u != request.max_new_tokens) fail("ArcLLM runtime generated-token count mismatch");

    // request close: reuse 0 evicts a resident image (runtime.cpp:508-517)
    if (q4_backend.has_sources())
        apply(cuda::decide_q4_down(profile1, request.request_within_validated_domain, 0u, runtime_state(),
                                   q4_backend.exec_family_bytes()));
    if (q4_backend.resident()) fail("ArcLLM runtime represented Q4 image still resident after request close");

    RuntimeStats& s = result.stats;
    s.prefill_dispatches = st.prefill_launches;
    s.prefill_submits = st.prefill_graph_launches;
    s.decode_dispatches_per_step = request.max_new_tokens > 1 ? st.decode_launches_per_step : 0u;
    s.decode_submits_per_step = request.max_new_tokens > 1 ? st.decode_graph_launches_per_step : 0u;
    s.decode_steps = st.decode_steps;
    s.route_a_steps = route_a_steps;
    s.route_b_steps = route_b_steps;
    s.acquire_events = acquire_events;
    s.evict_events = evict_events;
    const auto& c = q4_backend.counters();
    s.b_allocations = c.b_allocations;
    s.b_materializations = c.b_materializations;
    s.b_validations = c.b_validations;
    s.b_releases = c.b_releases;
    s.p1_calls = c.p1_calls;
    s.p3_calls = c.p3_calls;
    s.p0_calls = c.p0_calls;
    s.finite = true;
    check(arcllm_cuda_stream_synchronize(stream.s), "stream synchronize");
    return result;
}

}  // namespace arcllm::v1::runtime
