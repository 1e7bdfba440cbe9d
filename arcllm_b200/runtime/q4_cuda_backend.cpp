// Q4CudaBackend (include/arcllm/v1/q4_cuda_backend.h).
#include "arcllm/v1/q4_cuda_backend.h"

#include <sys/stat.h>

#include "arcllm_cuda.h"

namespace arcllm::v1::cuda {

using binding_v4::BackendStatus;

Q4CudaBackend::Q4CudaBackend(std::vector<Source> sources, std::uint32_t rows, std::uint32_t k,
                             std::string sidecar)
    : sources_(std::move(sources)), rows_(rows), k_(k), sidecar_(std::move(sidecar)) {}

Q4CudaBackend::~Q4CudaBackend() = default;

std::uint64_t Q4CudaBackend::exec_family_bytes() const noexcept {
    return std::uint64_t(sources_.size()) * rows_ * (k_ / 256u) * 148u;
}

bool Q4CudaBackend::p3_available() const noexcept {
    struct stat st{};
    return !sidecar_.empty() && ::stat(sidecar_.c_str(), &st) == 0 &&
           std::uint64_t(st.st_size) == exec_family_bytes();
}

const Q4CudaBackend::Source* Q4CudaBackend::find(std::uint32_t layer) const noexcept {
    for (const auto& s : sources_)
        if (s.layer == layer) return &s;
    return nullptr;
}

BackendStatus Q4CudaBackend::acquire(registry::AcquisitionPathId path, registry::PrimitiveId target,
                                     std::uint64_t residency_bytes,
                                     binding_v4::RepresentationHandle& out) noexcept {
    out = {};
    // Same precondition order as the Vulkan backend: wrong target or size, or
    // already resident, is a binding-state error; a missing or wrong-size
    // sidecar makes P3 unavailable; unknown paths are unavailable.
    if (target != kPrimitiveB || residency_bytes != exec_family_bytes()) return BackendStatus::INVALID_BINDING_STATE;
    if (resident_) return BackendStatus::INVALID_BINDING_STATE;
    if (path == kAcquireSecondary && !p3_available()) return BackendStatus::UNAVAILABLE;
    if (path != kAcquirePrimary && path != kAcquireSecondary && path != kAcquireTertiary)
        return BackendStatus::UNAVAILABLE;
    last_error_ = "EXEC148 representation (primitive B) is not provided by the CUDA backend";
    return BackendStatus::UNAVAILABLE;
}

BackendStatus Q4CudaBackend::validate(binding_v4::RepresentationHandle representation,
                                      registry::CapabilityId capability, registry::PrimitiveId target) noexcept {
    if (representation.opaque != 1ull || capability != kCapability || target != kPrimitiveB || !resident_)
        return BackendStatus::INVALID_BINDING_STATE;
    validated_ = false;
    return BackendStatus::VALIDATION_FAILED;
}

BackendStatus Q4CudaBackend::release(registry::PrimitiveId target,
                                     binding_v4::RepresentationHandle representation) noexcept {
    if (target != kPrimitiveB || representation.opaque != 1ull || !resident_)
        return BackendStatus::INVALID_BINDING_STATE;
    resident_ = false;
    validated_ = false;
    ++counters_.b_releases;
    return BackendStatus::OK;
}

BackendStatus Q4CudaBackend::resolve_primitive(registry::PrimitiveId primitive,
                                               binding_v4::PrimitiveHandle& out) noexcept {
    out = {};
    if (primitive == kPrimitiveA) {
        ++counters_.resolve_a;
        // Route A needs the CUDA library and a device; the Vulkan backend
        // checks for its shader file at this point instead.
        int n = 0;
        if (arcllm_cuda_abi_version() == 0 || arcllm_cuda_device_count(&n) != ARC_OK || n <= 0)
            return BackendStatus::PRIMITIVE_UNAVAILABLE;
        out = {primitive.value};
        return BackendStatus::OK;
    }
    if (primitive == kPrimitiveB) {
        ++counters_.resolve_b;
        if (!resident_ || !validated_) return BackendStatus::PRIMITIVE_UNAVAILABLE;
        return BackendStatus::PRIMITIVE_UNAVAILABLE;
    }
    return BackendStatus::PRIMITIVE_UNAVAILABLE;
}

int Q4CudaBackend::launch_ffn_down(binding_v4::PrimitiveHandle handle, std::uint32_t layer, const float* s,
                                   const float* residual, float* y, void* stream) const noexcept {
    if (handle.opaque != kPrimitiveA.value) return ARC_E_INVALID_ARGUMENT;
    const Source* src = find(layer);
    if (!src) return ARC_E_INVALID_ARGUMENT;
    return arcllm_cuda_matvec(ARC_GGML_Q4_K, src->device, rows_, k_, s, nullptr, 0.0f, nullptr, residual, y,
                              stream);
}

}  // namespace arcllm::v1::cuda
