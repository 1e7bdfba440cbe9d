// decide_q4_down (include/arcllm/v1/q4_down_policy.h).
#include "arcllm/v1/q4_down_policy.h"

namespace arcllm::v1::cuda {

namespace {

struct Path {
    registry::AcquisitionPathId id;
    std::uint32_t priority;
    std::uint64_t threshold[2];  // profile 0, profile 1
};

// registration_v2.cpp:37-49 (the warm-page-cache path is DISABLED_BY_EVIDENCE and never considered)
constexpr Path kPaths[] = {
    {kAcquirePrimary, 0u, {2u, 4u}},
    {kAcquireSecondary, 1u, {15u, 33u}},
    {kAcquireTertiary, 2u, {17u, 37u}},
};

Q4DownDecision route_a(Q4DownReason reason, bool preserve = false) {
    Q4DownDecision d;
    d.route = kPrimitiveA;
    d.reason = reason;
    d.preserve_existing_representation = preserve;
    return d;
}

}  // namespace

Q4DownDecision decide_q4_down(bool profile1, bool within_scope, std::uint64_t future_reuse, const Q4DownRuntime& rt,
                              std::uint64_t residency_bytes) noexcept {
    if (rt.b_resident) {  // engine :154-183 (B requires residency; lease always granted, execution available)
        if (!rt.b_identity_valid) {
            Q4DownDecision d = route_a(Q4DownReason::RESIDENT_PRIMITIVE_INVALID);
            d.lifecycle = Q4DownLifecycle::EVICT;
            return d;
        }
        if (future_reuse == 0) {
            Q4DownDecision d = route_a(Q4DownReason::NO_FUTURE_REUSE);
            d.lifecycle = Q4DownLifecycle::EVICT;
            return d;
        }
        if (!within_scope) return route_a(Q4DownReason::OUTSIDE_VALIDATED_DOMAIN, true);
        Q4DownDecision d;
        d.route = kPrimitiveB;
        d.reason = Q4DownReason::RESIDENT_PRIMITIVE_REUSED;
        d.preserve_existing_representation = true;
        return d;
    }
    if (!within_scope) return route_a(Q4DownReason::OUTSIDE_VALIDATED_DOMAIN);  // engine :192-197

    // candidate acquisition paths (engine :220-272): reuse-amortised, best = lowest priority meeting its threshold
    const Path* best = nullptr;
    const Path* best_below = nullptr;
    bool semantic_block = false;
    const bool available[3] = {rt.p1_available, rt.p3_available, rt.p0_available};
    for (int i = 0; i < 3; ++i) {
        if (!available[i]) continue;
        if (future_reuse == 0) {
            semantic_block = true;
            continue;
        }
        const Path& p = kPaths[i];
        if (future_reuse < p.threshold[profile1 ? 1 : 0]) {
            if (!best_below || p.priority < best_below->priority) best_below = &p;
            continue;
        }
        if (!best || p.priority < best->priority) best = &p;
    }
    if (best) {  // engine :274-287
        Q4DownDecision d;
        d.route = kPrimitiveB;
        d.lifecycle = Q4DownLifecycle::ACQUIRE;
        d.acquisition = best->id;
        d.reason = Q4DownReason::ACQUISITION_THRESHOLD_MET;
        d.threshold_units = best->threshold[profile1 ? 1 : 0];
        d.requested_residency_bytes = residency_bytes;
        d.require_post_acquisition_identity_validation = true;
        return d;
    }
    if (best_below) {  // engine :292-297
        Q4DownDecision d = route_a(Q4DownReason::BELOW_ALL_ACTIVE_THRESHOLDS);
        d.threshold_units = best_below->threshold[profile1 ? 1 : 0];
        return d;
    }
    if (semantic_block) return route_a(Q4DownReason::NO_FUTURE_REUSE);
    return route_a(Q4DownReason::NO_AVAILABLE_ACQUISITION_PATH);
}

}  // namespace arcllm::v1::cuda
