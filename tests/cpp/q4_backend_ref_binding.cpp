// Q4CudaBackend driven by the reference's OWN policy layer (TEST PROGRAM).
//
// Compiled (by oracle/build.py, into oracle/_ref/) against the reference's
// headers -- q4_cuda_backend.h then takes binding_v4::BackendAdapter from
// include/arcllm/v1/generic_backend_binding_v4.h of the ArcLLM checkout
// instead of the restated include/arcllm/v1/backend_adapter_v4.h -- and
// linked with the reference's policy engine, primitive registry, backend
// binding and Q4 FFN-down registration sources, plus libarcllm_runtime.so.
// It replays scenarios S1-S9 of the reference's Vulkan backend validation
// (src/arcllm_v1_q4_vulkan_backend_v4.cpp:661-841): every decision comes from
// policy_v4::evaluate and is carried out by binding_v4::apply_decision
// (src/arcllm_v1_generic_backend_binding_v4.cpp:52) on the CUDA backend.
// Weights: 14 Q4_K FFN-down layers of the Qwen2.5-7B shape (3584 x 18944,
// the registration's 549,527,552-byte EXEC148 family), filled on the GPU by
// the library's fixture stream.  Each routed primitive is executed
// (launch_ffn_down) and compared with the plain Q4_K matvec of the layer.
// argv[1]: a scratch directory for the P3 sidecar.  Needs a GPU.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <string>
#include <vector>

#include "arcllm/v1/generic_policy_engine_v4.h"
#include "arcllm/v1/q4_cuda_backend.h"
#include "arcllm_cuda.h"
#include "registrations/arcllm_v1_q4k_down_reference_registration_v2.h"

using namespace arcllm::v1;
namespace gp = policy_v4;
namespace bind = binding_v4;
namespace q4reg = reference_registration_v2;

static int failures = 0;
#define EXPECT(cond)                                                   \
    do {                                                               \
        if (!(cond)) {                                                 \
            std::printf("FAIL %s:%d %s\n", __FILE__, __LINE__, #cond); \
            ++failures;                                                \
        }                                                              \
    } while (0)

static const std::uint32_t kRows = 3584, kK = 18944, kLayers = 14;

static gp::PolicyDecision decide(const registry_v2::PrimitiveRegistry& reg, const cuda::Q4CudaBackend& b,
                                 std::uint64_t reuse, bool p1, bool p3, bool p0) {
    gp::PrimitiveRuntimeState prims[2]{};
    prims[0].primitive = q4reg::kPrimitiveA;
    prims[0].execution_available = prims[0].execution_ready = prims[0].residency_lease_granted = true;
    prims[1].primitive = q4reg::kPrimitiveB;
    prims[1].resident = b.resident();
    prims[1].identity_valid = b.validated();
    prims[1].execution_available = prims[1].execution_ready = prims[1].residency_lease_granted = true;
    gp::AcquisitionRuntimeState acq[3]{};
    acq[0].acquisition = q4reg::kAcquirePrimary;
    acq[0].available = p1;
    acq[1].acquisition = q4reg::kAcquireSecondary;
    acq[1].available = p3;
    acq[2].acquisition = q4reg::kAcquireTertiary;
    acq[2].available = p0;
    gp::PolicyRequest r{};
    r.capability = q4reg::kCapability;
    r.profile = q4reg::kProfile0;
    r.future_reuse_known = true;
    r.future_reuse_units = reuse;
    r.primitive_states = prims;
    r.primitive_state_count = 2;
    r.acquisition_states = acq;
    r.acquisition_state_count = 3;
    return gp::evaluate(reg, r);
}

// y = W_down(layer) s through the routed primitive against the plain Q4_K matvec
static bool component_ok(const cuda::Q4CudaBackend& b, bind::PrimitiveHandle h, std::uint32_t layer,
                         const void* w_layer, const float* s, float* y, float* yref) {
    if (b.launch_ffn_down(h, layer, s, nullptr, y, nullptr) != 0) return false;
    if (arcllm_cuda_matvec(ARC_GGML_Q4_K, w_layer, kRows, kK, s, nullptr, 0.f, nullptr, nullptr, yref, nullptr))
        return false;
    std::vector<float> a(kRows), r(kRows);
    if (arcllm_cuda_memcpy_d2h(a.data(), y, 4ull * kRows, nullptr) || arcllm_cuda_memcpy_d2h(r.data(), yref, 4ull * kRows, nullptr) ||
        arcllm_cuda_stream_synchronize(nullptr))
        return false;
    double num = 0, den = 0;
    for (std::uint32_t i = 0; i < kRows; ++i) {
        if (!std::isfinite(a[i])) return false;
        num += double(a[i] - r[i]) * double(a[i] - r[i]);
        den += double(r[i]) * double(r[i]);
    }
    return std::sqrt(num / den) <= 1e-5;
}

int main(int argc, char** argv) {
    if (argc < 2) return 64;
    const std::string sidecar = std::string(argv[1]) + "/exec148_family.bin";
    std::remove(sidecar.c_str());
    const std::uint64_t layer_bytes = std::uint64_t(kRows) * (kK / 256) * 144;
    void* w = nullptr;
    if (arcllm_cuda_malloc(layer_bytes * kLayers + 16, &w)) return 2;
    std::vector<std::uint8_t> host(layer_bytes * kLayers);
    std::vector<cuda::Q4CudaBackend::Source> src;
    for (std::uint32_t i = 0; i < kLayers; ++i) {
        auto* p = static_cast<std::uint8_t*>(w) + i * layer_bytes;
        if (arcllm_cuda_fill_q4k(p, 0, std::uint64_t(kRows) * (kK / 256), 0x5B00 + i, nullptr)) return 2;
        src.push_back({2u * i, p, host.data() + i * layer_bytes});  // layers 0, 2, 4, ...
    }
    if (arcllm_cuda_memcpy_d2h(host.data(), w, host.size(), nullptr) || arcllm_cuda_stream_synchronize(nullptr))
        return 2;
    void *s = nullptr, *y = nullptr, *yref = nullptr;
    if (arcllm_cuda_malloc(4ull * kK, &s) || arcllm_cuda_malloc(4ull * kRows, &y) ||
        arcllm_cuda_malloc(4ull * kRows, &yref) ||
        arcllm_cuda_fill_normal_f32(static_cast<float*>(s), 0, kK, 0x5C, 0.f, 1.f, nullptr))
        return 2;
    const float* sv = static_cast<const float*>(s);
    float* yv = static_cast<float*>(y);
    float* rv = static_cast<float*>(yref);

    cuda::Q4CudaBackend backend(src, kRows, kK, sidecar);
    EXPECT(backend.exec_family_bytes() == 549527552ull);
    registry_v2::PrimitiveRegistry registry;
    registry_v2::RegistryError rerr{};
    EXPECT(registry.add_bundle(q4reg::q4k_down_reference_bundle(), &rerr) == registry_v2::RegistryStatus::OK);
    bind::BindingState state{};
    auto apply = [&](const gp::PolicyDecision& d) {
        return bind::apply_decision(registry, q4reg::kCapability, d, backend, state);
    };

    // S1: reuse 1 routes A, nothing of B allocated or materialised
    const auto d1 = decide(registry, backend, 1, true, backend.p3_available(), true);
    EXPECT(d1.status == gp::PolicyStatus::OK && d1.route == q4reg::kPrimitiveA &&
           d1.lifecycle == gp::LifecycleAction::NONE);
    const auto a1 = apply(d1);
    EXPECT(a1.ready && a1.primitive.opaque == q4reg::kPrimitiveA.value);
    EXPECT(backend.counters().b_allocations == 0 && backend.counters().b_materializations == 0 && !backend.resident());
    EXPECT(component_ok(backend, a1.primitive, 0, src[0].device, sv, yv, rv));

    // S2: P1 unavailable at reuse 2: the policy stays on A, the backend tries nothing else
    const auto d2 = decide(registry, backend, 2, false, false, true);
    EXPECT(d2.status == gp::PolicyStatus::OK && d2.route == q4reg::kPrimitiveA &&
           d2.lifecycle == gp::LifecycleAction::NONE);
    const auto a2 = apply(d2);
    EXPECT(a2.ready && a2.primitive.opaque == q4reg::kPrimitiveA.value);
    EXPECT(backend.counters().b_allocations == 0 && backend.counters().p3_calls == 0 && backend.counters().p0_calls == 0);

    // S3: reuse 2 with P1: acquire (GPU materialisation), validate, route B
    const auto d3 = decide(registry, backend, 2, true, backend.p3_available(), true);
    EXPECT(d3.status == gp::PolicyStatus::OK && d3.route == q4reg::kPrimitiveB &&
           d3.lifecycle == gp::LifecycleAction::ACQUIRE && d3.acquisition == q4reg::kAcquirePrimary);
    const auto a3 = apply(d3);
    EXPECT(a3.ready && a3.primitive.opaque == q4reg::kPrimitiveB.value);
    EXPECT(backend.resident() && backend.validated() && backend.counters().b_allocations == 1 &&
           backend.counters().b_materializations == 1 && backend.counters().p1_calls == 1 &&
           backend.counters().b_validations == 1);
    EXPECT(component_ok(backend, a3.primitive, 6, src[3].device, sv, yv, rv));
    // keep the image as the P3 sidecar for S8
    {
        std::vector<std::uint8_t> img(backend.exec_family_bytes());
        EXPECT(arcllm_cuda_memcpy_d2h(img.data(), backend.exec_image(0), img.size(), nullptr) == 0);
        arcllm_cuda_stream_synchronize(nullptr);
        std::ofstream f(sidecar, std::ios::binary | std::ios::trunc);
        f.write(reinterpret_cast<const char*>(img.data()), std::streamsize(img.size()));
    }

    // S4: resident B is reused with no re-acquisition
    const auto before = backend.counters();
    const auto d4 = decide(registry, backend, 1, true, backend.p3_available(), true);
    EXPECT(d4.status == gp::PolicyStatus::OK && d4.route == q4reg::kPrimitiveB &&
           d4.lifecycle == gp::LifecycleAction::NONE);
    const auto a4 = apply(d4);
    EXPECT(a4.ready && a4.primitive.opaque == q4reg::kPrimitiveB.value);
    EXPECT(backend.counters().b_allocations == before.b_allocations &&
           backend.counters().b_materializations == before.b_materializations);

    // S5: known zero reuse evicts B and routes A
    const auto d5 = decide(registry, backend, 0, true, backend.p3_available(), true);
    EXPECT(d5.status == gp::PolicyStatus::OK && d5.route == q4reg::kPrimitiveA &&
           d5.lifecycle == gp::LifecycleAction::EVICT);
    const auto a5 = apply(d5);
    EXPECT(a5.ready && a5.primitive.opaque == q4reg::kPrimitiveA.value);
    EXPECT(!backend.resident() && backend.counters().b_releases == 1);

    // S6: the tertiary P0 (CPU materialisation) chosen by the policy, never by a backend retry
    const auto d6 = decide(registry, backend, 17, false, false, true);
    EXPECT(d6.status == gp::PolicyStatus::OK && d6.route == q4reg::kPrimitiveB &&
           d6.lifecycle == gp::LifecycleAction::ACQUIRE && d6.acquisition == q4reg::kAcquireTertiary);
    const auto a6 = apply(d6);
    EXPECT(a6.ready && a6.primitive.opaque == q4reg::kPrimitiveB.value);
    EXPECT(backend.counters().p0_calls == 1 && backend.counters().b_allocations == 2 &&
           backend.counters().b_materializations == 2 && backend.counters().b_validations == 2);
    EXPECT(component_ok(backend, a6.primitive, 26, src[13].device, sv, yv, rv));

    // S7: final eviction
    const auto d7 = decide(registry, backend, 0, false, false, true);
    const auto a7 = apply(d7);
    EXPECT(a7.ready && a7.primitive.opaque == q4reg::kPrimitiveA.value && !backend.resident() &&
           backend.counters().b_releases == 2);

    // S8/S9: with the canonical sidecar present, P3 (cold read) chosen by the policy, executed once, evicted
    EXPECT(backend.p3_available());
    const auto d8 = decide(registry, backend, 15, false, true, true);
    EXPECT(d8.status == gp::PolicyStatus::OK && d8.route == q4reg::kPrimitiveB &&
           d8.lifecycle == gp::LifecycleAction::ACQUIRE && d8.acquisition == q4reg::kAcquireSecondary);
    const auto a8 = apply(d8);
    EXPECT(a8.ready && a8.primitive.opaque == q4reg::kPrimitiveB.value);
    EXPECT(backend.counters().p3_calls == 1 && backend.counters().b_allocations == 3 &&
           backend.counters().b_materializations == 3 && backend.counters().b_validations == 3);
    EXPECT(component_ok(backend, a8.primitive, 12, src[6].device, sv, yv, rv));
    const auto d9 = decide(registry, backend, 0, false, true, true);
    const auto a9 = apply(d9);
    EXPECT(a9.ready && a9.primitive.opaque == q4reg::kPrimitiveA.value && !backend.resident() &&
           backend.counters().b_releases == 3);

    // a corrupted sidecar: P3 acquires, identity validation fails, apply_decision releases it
    {
        std::fstream f(sidecar, std::ios::binary | std::ios::in | std::ios::out);
        f.seekp(1000);
        f.put('\x5A');
    }
    const auto d10 = decide(registry, backend, 15, false, true, true);
    const auto a10 = apply(d10);
    EXPECT(!a10.ready && a10.backend_status == bind::BackendStatus::VALIDATION_FAILED &&
           a10.cleanup_status == bind::BackendStatus::OK && !backend.resident());

    std::remove(sidecar.c_str());
    arcllm_cuda_free(w);
    arcllm_cuda_free(s);
    arcllm_cuda_free(y);
    arcllm_cuda_free(yref);
    const auto& c = backend.counters();
    std::printf("counters: alloc %llu mat %llu val %llu rel %llu p1 %llu p3 %llu p0 %llu resolve A %llu B %llu\n",
                (unsigned long long)c.b_allocations, (unsigned long long)c.b_materializations,
                (unsigned long long)c.b_validations, (unsigned long long)c.b_releases, (unsigned long long)c.p1_calls,
                (unsigned long long)c.p3_calls, (unsigned long long)c.p0_calls, (unsigned long long)c.resolve_a,
                (unsigned long long)c.resolve_b);
    std::printf("q4_backend_ref_binding: %d failure(s)\n", failures);
    return failures ? 1 : 0;
}
