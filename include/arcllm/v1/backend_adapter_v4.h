// The backend-binding interface of ArcLLM's generic policy layer, restated
// with the same names, layouts and status values as the reference
// (include/arcllm/v1/primitive_registry_model.h:7-32 for the opaque ids,
// include/arcllm/v1/generic_backend_binding_v4.h:16-53 for the handles,
// BackendStatus and BackendAdapter), so a backend written against it -- the
// CUDA Q4 backend here -- compiles unchanged against the reference headers and
// plugs into binding_v4::apply_decision.  Only the types a backend needs are
// declared; the registry and the policy engine themselves stay in the
// reference's policy layer.
#pragma once
#include <cstdint>

namespace arcllm::v1::registry {

template <typename Tag>
struct OpaqueId {
    std::uint64_t value = 0;
    constexpr explicit operator bool() const noexcept { return value != 0; }
    friend constexpr bool operator==(OpaqueId a, OpaqueId b) noexcept { return a.value == b.value; }
    friend constexpr bool operator!=(OpaqueId a, OpaqueId b) noexcept { return !(a == b); }
};

struct CapabilityTag {};
struct PrimitiveTag {};
struct AcquisitionPathTag {};

using CapabilityId = OpaqueId<CapabilityTag>;
using PrimitiveId = OpaqueId<PrimitiveTag>;
using AcquisitionPathId = OpaqueId<AcquisitionPathTag>;

}  // namespace arcllm::v1::registry

namespace arcllm::v1::registry_v2 {
using registry::AcquisitionPathId;
using registry::CapabilityId;
using registry::PrimitiveId;
}  // namespace arcllm::v1::registry_v2

namespace arcllm::v1::binding_v4 {

using registry_v2::AcquisitionPathId;
using registry_v2::CapabilityId;
using registry_v2::PrimitiveId;

struct RepresentationHandle {
    std::uint64_t opaque = 0;
    constexpr explicit operator bool() const noexcept { return opaque != 0; }
};

struct PrimitiveHandle {
    std::uint64_t opaque = 0;
    constexpr explicit operator bool() const noexcept { return opaque != 0; }
};

enum class BackendStatus : std::uint8_t {
    OK = 0,
    UNAVAILABLE = 1,
    RESOURCE_DENIED = 2,
    ACQUISITION_FAILED = 3,
    VALIDATION_FAILED = 4,
    RELEASE_FAILED = 5,
    PRIMITIVE_UNAVAILABLE = 6,
    INVALID_BINDING_STATE = 7
};

class BackendAdapter {
public:
    virtual ~BackendAdapter() = default;
    virtual BackendStatus acquire(AcquisitionPathId path, PrimitiveId target, std::uint64_t residency_bytes,
                                  RepresentationHandle& out_representation) noexcept = 0;
    virtual BackendStatus validate(RepresentationHandle representation, CapabilityId capability,
                                   PrimitiveId target) noexcept = 0;
    virtual BackendStatus release(PrimitiveId target, RepresentationHandle representation) noexcept = 0;
    virtual BackendStatus resolve_primitive(PrimitiveId primitive, PrimitiveHandle& out_primitive) noexcept = 0;
};

}  // namespace arcllm::v1::binding_v4
