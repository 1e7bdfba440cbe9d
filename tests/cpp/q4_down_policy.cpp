// Route decisions of the Q4 FFN-down policy (TEST PROGRAM): the reference
// engine's outcomes for the registered bundle (reuse thresholds P1 2/4,
// P3 15/33, P0 17/37 for profiles 0/1; src/arcllm_v1_generic_policy_engine_v4.cpp).
#include <cstdio>

#include "arcllm/v1/q4_down_policy.h"

using namespace arcllm::v1;
using cuda::Q4DownLifecycle;
using cuda::Q4DownReason;

static int failures = 0;
#define EXPECT(cond)                                                   \
    do {                                                               \
        if (!(cond)) {                                                 \
            std::printf("FAIL %s:%d %s\n", __FILE__, __LINE__, #cond); \
            ++failures;                                                \
        }                                                              \
    } while (0)

static cuda::Q4DownDecision D(bool p1, bool scope, std::uint64_t reuse, cuda::Q4DownRuntime rt = {}) {
    return cuda::decide_q4_down(p1, scope, reuse, rt, 1000);
}

int main() {
    // not resident, inside the validated domain: P1 once reuse reaches its threshold
    auto d = D(false, true, 1);
    EXPECT(d.route == cuda::kPrimitiveA && d.reason == Q4DownReason::BELOW_ALL_ACTIVE_THRESHOLDS && d.threshold_units == 2);
    d = D(false, true, 2);
    EXPECT(d.route == cuda::kPrimitiveB && d.lifecycle == Q4DownLifecycle::ACQUIRE && d.acquisition == cuda::kAcquirePrimary);
    EXPECT(d.reason == Q4DownReason::ACQUISITION_THRESHOLD_MET && d.threshold_units == 2);
    EXPECT(d.requested_residency_bytes == 1000 && d.require_post_acquisition_identity_validation);
    d = D(true, true, 3);
    EXPECT(d.route == cuda::kPrimitiveA && d.threshold_units == 4);
    d = D(true, true, 4);
    EXPECT(d.lifecycle == Q4DownLifecycle::ACQUIRE && d.acquisition == cuda::kAcquirePrimary && d.threshold_units == 4);
    // zero future reuse: nothing to amortise
    d = D(false, true, 0);
    EXPECT(d.route == cuda::kPrimitiveA && d.reason == Q4DownReason::NO_FUTURE_REUSE && d.lifecycle == Q4DownLifecycle::NONE);
    // outside the validated domain: always A
    d = D(false, false, 100);
    EXPECT(d.route == cuda::kPrimitiveA && d.reason == Q4DownReason::OUTSIDE_VALIDATED_DOMAIN);
    // P1 unavailable: P3 (priority 1) when its sidecar exists and reuse >= 15, else P0 at >= 17
    cuda::Q4DownRuntime no_p1;
    no_p1.p1_available = false;
    no_p1.p3_available = true;
    d = D(false, true, 14, no_p1);
    EXPECT(d.route == cuda::kPrimitiveA && d.threshold_units == 15);
    d = D(false, true, 15, no_p1);
    EXPECT(d.acquisition == cuda::kAcquireSecondary);
    d = D(false, true, 20, no_p1);
    EXPECT(d.acquisition == cuda::kAcquireSecondary);  // lower priority number wins over P0
    no_p1.p3_available = false;
    d = D(false, true, 16, no_p1);
    EXPECT(d.route == cuda::kPrimitiveA && d.reason == Q4DownReason::BELOW_ALL_ACTIVE_THRESHOLDS && d.threshold_units == 17);
    d = D(false, true, 17, no_p1);
    EXPECT(d.acquisition == cuda::kAcquireTertiary);
    d = D(true, true, 36, no_p1);
    EXPECT(d.route == cuda::kPrimitiveA && d.threshold_units == 37);
    no_p1.p0_available = false;
    d = D(false, true, 100, no_p1);
    EXPECT(d.route == cuda::kPrimitiveA && d.reason == Q4DownReason::NO_AVAILABLE_ACQUISITION_PATH);
    // resident image
    cuda::Q4DownRuntime res;
    res.b_resident = true;
    res.b_identity_valid = true;
    d = D(false, true, 5, res);
    EXPECT(d.route == cuda::kPrimitiveB && d.reason == Q4DownReason::RESIDENT_PRIMITIVE_REUSED && d.lifecycle == Q4DownLifecycle::NONE);
    EXPECT(d.preserve_existing_representation);
    d = D(false, true, 0, res);
    EXPECT(d.route == cuda::kPrimitiveA && d.lifecycle == Q4DownLifecycle::EVICT && d.reason == Q4DownReason::NO_FUTURE_REUSE);
    d = D(false, false, 5, res);
    EXPECT(d.route == cuda::kPrimitiveA && d.lifecycle == Q4DownLifecycle::NONE && d.preserve_existing_representation);
    res.b_identity_valid = false;
    d = D(false, true, 5, res);
    EXPECT(d.route == cuda::kPrimitiveA && d.lifecycle == Q4DownLifecycle::EVICT &&
           d.reason == Q4DownReason::RESIDENT_PRIMITIVE_INVALID);
    std::printf("q4_down_policy: %d failure(s)\n", failures);
    return failures ? 1 : 0;
}
