// Route selection for the Q4 FFN-down capability: the decision the
// reference's generic policy engine takes for the bundle registered in
// src/registrations/arcllm_v1_q4k_down_reference_registration_v2.cpp:30-57
// (preferred primitive B = EXEC148 image, fallback A = plain Q4_K matvec;
// acquisition paths P1 GPU-in-place / P3 cold sidecar / P0 CPU, priorities
// 0/1/2, reuse thresholds 2/15/17 tokens under profile 0 and 4/33/37 under
// profile 1; lifecycle evicts on identity loss or zero future reuse and keeps
// the image outside the validated domain), restated from
// src/arcllm_v1_generic_policy_engine_v4.cpp:103-317 for that bundle.  The
// reason and lifecycle values are the engine's (policy_v4::PolicyReason,
// policy_v4::LifecycleAction), so logs and tests compare one-to-one.
#pragma once
#include <cstdint>

#include "arcllm/v1/q4_cuda_backend.h"

namespace arcllm::v1::cuda {

enum class Q4DownLifecycle : std::uint8_t { NONE = 0, ACQUIRE = 1, EVICT = 2 };

enum class Q4DownReason : std::uint8_t {
    FALLBACK_ONLY = 0,
    OUTSIDE_VALIDATED_DOMAIN = 1,
    RESIDENT_PRIMITIVE_INVALID = 3,
    NO_FUTURE_REUSE = 6,
    RESIDENT_PRIMITIVE_REUSED = 7,
    NO_AVAILABLE_ACQUISITION_PATH = 10,
    BELOW_ALL_ACTIVE_THRESHOLDS = 11,
    ACQUISITION_THRESHOLD_MET = 12
};

// What the runtime knows about primitive B and the acquisition paths.
struct Q4DownRuntime {
    bool b_resident = false;
    bool b_identity_valid = false;
    bool p1_available = true;   // GPU materialisation from the resident Q4_K weights
    bool p3_available = false;  // sidecar file of the right size
    bool p0_available = true;   // CPU materialisation from the mapped file
};

struct Q4DownDecision {
    registry::PrimitiveId route{};
    Q4DownLifecycle lifecycle = Q4DownLifecycle::NONE;
    registry::AcquisitionPathId acquisition{};
    Q4DownReason reason = Q4DownReason::FALLBACK_ONLY;
    std::uint64_t threshold_units = 0;
    std::uint64_t requested_residency_bytes = 0;
    bool preserve_existing_representation = false;
    bool require_post_acquisition_identity_validation = false;
};

// profile1: EvidenceProfile::PROFILE_1 (else PROFILE_0); within_scope: the
// request lies inside the validated domain; future_reuse: decode steps still
// to run after this one; residency_bytes: size of the B image.
Q4DownDecision decide_q4_down(bool profile1, bool within_scope, std::uint64_t future_reuse, const Q4DownRuntime& rt,
                              std::uint64_t residency_bytes) noexcept;

}  // namespace arcllm::v1::cuda
