// Status semantics of Q4CudaBackend (TEST PROGRAM): the precondition order of
// the reference's Vulkan backend (src/arcllm_v1_q4_vulkan_backend_v4_runtime.h
// :210-345) on every path that needs no GPU.  argv[1] = a scratch directory
// for the sidecar files, argv[2] = "gpu" when a device is present.
#include <cstdio>
#include <fstream>
#include <string>

#include "arcllm/v1/q4_cuda_backend.h"

using namespace arcllm::v1;
using binding_v4::BackendStatus;

static int failures = 0;
#define EXPECT(cond)                                                   \
    do {                                                               \
        if (!(cond)) {                                                 \
            std::printf("FAIL %s:%d %s\n", __FILE__, __LINE__, #cond); \
            ++failures;                                                \
        }                                                              \
    } while (0)

int main(int argc, char** argv) {
    if (argc < 3) return 64;
    const std::string dir = argv[1];
    const bool gpu = std::string(argv[2]) == "gpu";
    const std::uint32_t rows = 256, k = 512;
    // two Q4 down layers; device pointers are never dereferenced on these paths
    std::vector<cuda::Q4CudaBackend::Source> src = {{3, nullptr}, {4, nullptr}};
    const std::string sidecar = dir + "/exec148.bin";
    cuda::Q4CudaBackend b(src, rows, k, sidecar);
    const std::uint64_t bytes = 2ull * rows * (k / 256) * 148;
    EXPECT(b.exec_family_bytes() == bytes);
    EXPECT(!b.resident() && !b.validated());

    binding_v4::RepresentationHandle rep{};
    // wrong target / wrong residency size -> INVALID_BINDING_STATE, handle cleared
    rep.opaque = 77;
    EXPECT(b.acquire(cuda::kAcquirePrimary, cuda::kPrimitiveA, bytes, rep) == BackendStatus::INVALID_BINDING_STATE);
    EXPECT(rep.opaque == 0);
    EXPECT(b.acquire(cuda::kAcquirePrimary, cuda::kPrimitiveB, bytes + 1, rep) == BackendStatus::INVALID_BINDING_STATE);
    // P3 without a sidecar, or with a wrong-size one -> UNAVAILABLE
    EXPECT(!b.p3_available());
    EXPECT(b.acquire(cuda::kAcquireSecondary, cuda::kPrimitiveB, bytes, rep) == BackendStatus::UNAVAILABLE);
    { std::ofstream(sidecar, std::ios::binary) << "short"; }
    EXPECT(!b.p3_available());
    EXPECT(b.acquire(cuda::kAcquireSecondary, cuda::kPrimitiveB, bytes, rep) == BackendStatus::UNAVAILABLE);
    {
        std::ofstream f(sidecar, std::ios::binary | std::ios::trunc);
        f.seekp(std::streamoff(bytes - 1));
        f.put('\0');
    }
    EXPECT(b.p3_available());
    // the disabled warm path and unknown paths -> UNAVAILABLE
    EXPECT(b.acquire(cuda::kAcquireDisabledWarm, cuda::kPrimitiveB, bytes, rep) == BackendStatus::UNAVAILABLE);
    EXPECT(b.acquire(registry::AcquisitionPathId{0x1234}, cuda::kPrimitiveB, bytes, rep) ==
           BackendStatus::UNAVAILABLE);
    // P1 / P0 on sources that cannot be materialised (no device or null
    // weights, no host copy): ACQUISITION_FAILED, nothing left resident
    EXPECT(b.acquire(cuda::kAcquirePrimary, cuda::kPrimitiveB, bytes, rep) == BackendStatus::ACQUISITION_FAILED);
    EXPECT(rep.opaque == 0 && !b.resident());
    EXPECT(b.acquire(cuda::kAcquireTertiary, cuda::kPrimitiveB, bytes, rep) == BackendStatus::ACQUISITION_FAILED);
    EXPECT(!b.last_error().empty());
    EXPECT(!b.resident());
    // P3 with a sidecar of the right size: on a GPU the image is read and
    // resident (handle 1), identity validation against the null sources
    // fails, release frees it; without a GPU the allocation fails
    const BackendStatus p3 = b.acquire(cuda::kAcquireSecondary, cuda::kPrimitiveB, bytes, rep);
    if (gpu) {
        EXPECT(p3 == BackendStatus::OK && rep.opaque == 1 && b.resident() && !b.validated());
        EXPECT(b.acquire(cuda::kAcquirePrimary, cuda::kPrimitiveB, bytes, rep) == BackendStatus::INVALID_BINDING_STATE);
        rep.opaque = 1;
        EXPECT(b.validate(rep, cuda::kCapability, cuda::kPrimitiveB) == BackendStatus::VALIDATION_FAILED);
        EXPECT(!b.validated());
        EXPECT(b.release(cuda::kPrimitiveB, rep) == BackendStatus::OK);
        EXPECT(!b.resident());
    } else {
        EXPECT(p3 == BackendStatus::ACQUISITION_FAILED && !b.resident());
    }
    // validate / release without a resident image -> INVALID_BINDING_STATE
    EXPECT(b.validate({1}, cuda::kCapability, cuda::kPrimitiveB) == BackendStatus::INVALID_BINDING_STATE);
    EXPECT(b.validate({0}, cuda::kCapability, cuda::kPrimitiveB) == BackendStatus::INVALID_BINDING_STATE);
    EXPECT(b.release(cuda::kPrimitiveB, {1}) == BackendStatus::INVALID_BINDING_STATE);
    EXPECT(b.release(cuda::kPrimitiveA, {1}) == BackendStatus::INVALID_BINDING_STATE);
    // primitives
    binding_v4::PrimitiveHandle h{};
    h.opaque = 9;
    EXPECT(b.resolve_primitive(cuda::kPrimitiveB, h) == BackendStatus::PRIMITIVE_UNAVAILABLE);
    EXPECT(h.opaque == 0);
    EXPECT(b.resolve_primitive(registry::PrimitiveId{0xDEAD}, h) == BackendStatus::PRIMITIVE_UNAVAILABLE);
    const BackendStatus ra = b.resolve_primitive(cuda::kPrimitiveA, h);
    if (gpu) {
        EXPECT(ra == BackendStatus::OK);
        EXPECT(h.opaque == cuda::kPrimitiveA.value);
    } else {
        EXPECT(ra == BackendStatus::PRIMITIVE_UNAVAILABLE);
    }
    // a route-A launch for a layer the backend does not hold is refused before any launch
    EXPECT(b.launch_ffn_down({cuda::kPrimitiveA.value}, 5, nullptr, nullptr, nullptr, nullptr) != 0);
    EXPECT(b.launch_ffn_down({cuda::kPrimitiveB.value}, 3, nullptr, nullptr, nullptr, nullptr) != 0);
    const auto& c = b.counters();
    EXPECT(c.resolve_a == 1 && c.resolve_b == 1);
    EXPECT(c.p1_calls == (gpu ? 1u : 0u) && c.p0_calls == (gpu ? 1u : 0u) && c.p3_calls == (gpu ? 1u : 0u));
    EXPECT(c.b_materializations == (gpu ? 1u : 0u) && c.b_releases == (gpu ? 1u : 0u));
    EXPECT(c.b_validations == (gpu ? 1u : 0u));
    std::printf("q4_backend_status: %d failure(s)\n", failures);
    return failures ? 1 : 0;
}
