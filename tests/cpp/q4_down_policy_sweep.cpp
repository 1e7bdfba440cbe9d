// Decisions of decide_q4_down over a sweep of its inputs (TEST PROGRAM): one
// line per input, "profile1 scope reuse resident valid p1 p3 p0 : route
// lifecycle acquisition reason threshold bytes flags", compared by
// tests/test_policy_pin_cpu.py with the reference's own policy engine
// (src/arcllm_v1_generic_policy_engine_v4.cpp:103-317 with the Q4 FFN-down
// registration) on the same inputs.
#include <cstdio>

#include "arcllm/v1/q4_down_policy.h"

using namespace arcllm::v1;

int main() {
    const unsigned long long kBytes = 549527552ull;  // the registration's residency bytes of primitive B
    for (int p1 = 0; p1 < 2; ++p1)
        for (int scope = 0; scope < 2; ++scope)
            for (unsigned reuse = 0; reuse <= 40; ++reuse)
                for (int res = 0; res < 2; ++res)
                    for (int valid = 0; valid < 2; ++valid)
                        for (int avail = 0; avail < 8; ++avail) {
                            cuda::Q4DownRuntime rt;
                            rt.b_resident = res != 0;
                            rt.b_identity_valid = valid != 0;
                            rt.p1_available = (avail & 1) != 0;
                            rt.p3_available = (avail & 2) != 0;
                            rt.p0_available = (avail & 4) != 0;
                            const cuda::Q4DownDecision d = cuda::decide_q4_down(p1 != 0, scope != 0, reuse, rt, kBytes);
                            std::printf("%d %d %u %d %d %d %d %d : %llu %u %llu %u %llu %llu %u\n", p1, scope, reuse,
                                        res, valid, avail & 1, (avail >> 1) & 1, (avail >> 2) & 1,
                                        (unsigned long long)d.route.value, (unsigned)d.lifecycle,
                                        (unsigned long long)d.acquisition.value, (unsigned)d.reason,
                                        (unsigned long long)d.threshold_units,
                                        (unsigned long long)d.requested_residency_bytes,
                                        (d.preserve_existing_representation ? 1u : 0u) |
                                            (d.require_post_acquisition_identity_validation ? 2u : 0u));
                        }
    return 0;
}
