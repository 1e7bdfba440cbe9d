/*
 * C-ABI export of the reference's OWN generic policy engine for the Q4
 * FFN-down bundle, compiled in place from the ArcLLM sources (nothing is
 * copied: the files are #included from the path given with -I by
 * oracle/build.py, the output goes to oracle/_ref/).  TEST INFRASTRUCTURE
 * ONLY: pins the restated route selection (arcllm_b200/runtime/
 * q4_down_policy.cpp) decision for decision.
 *
 *   src/arcllm_v1_generic_policy_engine_v4.cpp   -- policy_v4::evaluate (103-317)
 *   src/arcllm_v1_primitive_registry_v2.cpp      -- registry_v2::PrimitiveRegistry
 *   src/registrations/arcllm_v1_q4k_down_reference_registration_v2.cpp
 *                                                 -- q4k_down_reference_bundle (54)
 */
#include <cstdint>

#include "arcllm_v1_generic_policy_engine_v4.cpp"
#include "arcllm_v1_primitive_registry_v2.cpp"
#include "registrations/arcllm_v1_q4k_down_reference_registration_v2.cpp"

namespace {
namespace P = arcllm::v1::policy_v4;
namespace R = arcllm::v1::reference_registration_v2;
}  // namespace

extern "C" {

/* in[0] profile 1 (else 0), in[1] request inside the validated domain,
 * in[2] future reuse units (known), in[3] B resident, in[4] B identity valid,
 * in[5..7] P1 / P3 / P0 available.  Model loaded, acquisition allowed,
 * both primitives executable and ready, residency lease granted (the runtime
 * conditions of generate()).  out: status, route, lifecycle, acquisition,
 * reason, threshold units, requested residency bytes,
 * preserve | (require validation << 1).  Returns the registry status. */
int ref_q4_down_evaluate(const uint64_t* in, uint64_t* out) {
    static arcllm::v1::registry_v2::PrimitiveRegistry reg;
    static int reg_status = static_cast<int>(reg.add_bundle(R::q4k_down_reference_bundle()));
    if (reg_status != 0) return reg_status;
    P::PrimitiveRuntimeState prims[2]{};
    prims[0].primitive = R::kPrimitiveA;
    prims[0].execution_available = prims[0].execution_ready = prims[0].residency_lease_granted = true;
    prims[1].primitive = R::kPrimitiveB;
    prims[1].resident = in[3] != 0;
    prims[1].identity_valid = in[4] != 0;
    prims[1].execution_available = prims[1].execution_ready = prims[1].residency_lease_granted = true;
    P::AcquisitionRuntimeState acq[3]{};
    acq[0].acquisition = R::kAcquirePrimary;
    acq[0].available = in[5] != 0;
    acq[1].acquisition = R::kAcquireSecondary;
    acq[1].available = in[6] != 0;
    acq[2].acquisition = R::kAcquireTertiary;
    acq[2].available = in[7] != 0;
    P::PolicyRequest r{};
    r.capability = R::kCapability;
    r.profile = in[0] ? R::kProfile1 : R::kProfile0;
    r.request_within_capability_evidence_scope = in[1] != 0;
    r.model_loaded = true;
    r.future_reuse_known = true;
    r.future_reuse_units = in[2];
    r.acquisition_allowed = true;
    r.primitive_states = prims;
    r.primitive_state_count = 2;
    r.acquisition_states = acq;
    r.acquisition_state_count = 3;
    const P::PolicyDecision d = P::evaluate(reg, r);
    out[0] = static_cast<uint64_t>(d.status);
    out[1] = d.route.value;
    out[2] = static_cast<uint64_t>(d.lifecycle);
    out[3] = d.acquisition.value;
    out[4] = static_cast<uint64_t>(d.reason);
    out[5] = d.threshold_units;
    out[6] = d.requested_residency_bytes;
    out[7] = (d.preserve_existing_representation ? 1u : 0u) | (d.require_post_acquisition_identity_validation ? 2u : 0u);
    return 0;
}

}  // extern "C"
