// Q4CudaBackend: the CUDA implementation of the ArcLLM Q4_K FFN-down backend.
//
// It implements binding_v4::BackendAdapter with the status semantics of the
// reference's Vulkan backend (src/arcllm_v1_q4_vulkan_backend_v4_runtime.h:
// acquire :210-275, validate :277-305, release :307-321, resolve_primitive
// :323-345) so the reference's policy layer (binding_v4::apply_decision) can
// drive it unchanged.  Primitive A is the plain Q4_K split-K matvec over the
// GGUF layout; primitive B is the EXEC148 image of all Q4_K FFN-down layers
// (148 bytes per super-block), acquired by GPU materialisation (P1), a cold
// sidecar read (P3) or CPU materialisation (P0), and validated block by block
// against its Q4_K source (canonical tuples identical).  launch_ffn_down is
// the counterpart of append_ffn_down_op (:347-385).
#pragma once
#include <cstdint>
#include <string>
#include <vector>

#if defined(ARCLLM_BINDING_FROM_REFERENCE)
// a program built against the reference's own policy layer takes the adapter
// interface from there (same names, layouts and values as the restatement)
#include "arcllm/v1/generic_backend_binding_v4.h"
#else
#include "arcllm/v1/backend_adapter_v4.h"
#endif

namespace arcllm::v1::cuda {

// Ids of the Q4 FFN-down registration bundle
// (src/registrations/arcllm_v1_q4k_down_reference_registration_v2.h:12-19).
inline constexpr registry::CapabilityId kCapability{0x00010001ull};
inline constexpr registry::PrimitiveId kPrimitiveA{0xA001ull};
inline constexpr registry::PrimitiveId kPrimitiveB{0xB001ull};
inline constexpr registry::AcquisitionPathId kAcquirePrimary{0xC101ull};
inline constexpr registry::AcquisitionPathId kAcquireSecondary{0xC102ull};
inline constexpr registry::AcquisitionPathId kAcquireTertiary{0xC103ull};
inline constexpr registry::AcquisitionPathId kAcquireDisabledWarm{0xC104ull};

struct BackendCounters {
    std::uint64_t b_allocations = 0;
    std::uint64_t b_materializations = 0;
    std::uint64_t b_validations = 0;
    std::uint64_t b_releases = 0;
    std::uint64_t p1_calls = 0;
    std::uint64_t p3_calls = 0;
    std::uint64_t p0_calls = 0;
    std::uint64_t resolve_a = 0;
    std::uint64_t resolve_b = 0;
};

class Q4CudaBackend final : public binding_v4::BackendAdapter {
public:
    // One Q4_K ffn_down weight routed through this backend.
    struct Source {
        std::uint32_t layer = 0;
        const void* device = nullptr;         // Q4_K rows in device memory, 16-byte aligned
        const std::uint8_t* host = nullptr;  // the same bytes in host memory (P0; may be null)
    };
    // rows x k is the shape of every source (hidden x ffn); sidecar is the
    // optional pre-materialised image path (acquisition P3).
    Q4CudaBackend(std::vector<Source> sources, std::uint32_t rows, std::uint32_t k, std::string sidecar);
    ~Q4CudaBackend() override;
    Q4CudaBackend(const Q4CudaBackend&) = delete;
    Q4CudaBackend& operator=(const Q4CudaBackend&) = delete;

    binding_v4::BackendStatus acquire(registry::AcquisitionPathId path, registry::PrimitiveId target,
                                      std::uint64_t residency_bytes,
                                      binding_v4::RepresentationHandle& out) noexcept override;
    binding_v4::BackendStatus validate(binding_v4::RepresentationHandle representation,
                                       registry::CapabilityId capability,
                                       registry::PrimitiveId target) noexcept override;
    binding_v4::BackendStatus release(registry::PrimitiveId target,
                                      binding_v4::RepresentationHandle representation) noexcept override;
    binding_v4::BackendStatus resolve_primitive(registry::PrimitiveId primitive,
                                                binding_v4::PrimitiveHandle& out) noexcept override;

    // Enqueue y = W_down(layer) * s (+ residual) on `stream` with the primitive
    // `handle` resolved above.  Returns an arcllm_cuda status (0 = OK).
    int launch_ffn_down(binding_v4::PrimitiveHandle handle, std::uint32_t layer, const float* s,
                        const float* residual, float* y, void* stream) const noexcept;

    // Bytes of the EXEC148 image for all sources (148 B per Q4_K super-block).
    std::uint64_t exec_family_bytes() const noexcept;
    // Device address of `layer`'s slot in the resident EXEC148 image (null if
    // the image is not resident or the layer is not a source).
    const void* exec_image(std::uint32_t layer) const noexcept;
    bool has_sources() const noexcept { return !sources_.empty(); }
    bool resident() const noexcept { return resident_; }
    bool validated() const noexcept { return validated_; }
    bool p3_available() const noexcept;
    const BackendCounters& counters() const noexcept { return counters_; }
    const std::string& last_error() const noexcept { return last_error_; }

private:
    const Source* find(std::uint32_t layer) const noexcept;
    std::uint64_t layer_bytes() const noexcept { return std::uint64_t(rows_) * (k_ / 256u) * 148u; }
    void free_image() noexcept;
    std::vector<Source> sources_;
    std::uint32_t rows_, k_;
    std::string sidecar_;
    void* image_ = nullptr;  // device memory of the EXEC148 image
    bool resident_ = false;
    bool validated_ = false;
    BackendCounters counters_{};
    std::string last_error_;
};

}  // namespace arcllm::v1::cuda
