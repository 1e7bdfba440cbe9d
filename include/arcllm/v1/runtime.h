// Public runtime API of ArcLLM, kept declaration-for-declaration identical to
// include/arcllm/v1/runtime.h of the reference (RunRequest :13-23,
// RuntimeStats :25-46, RunResult :48-51, generate :57) so callers switch
// implementations without source changes.  This implementation runs the
// decode hot path on a B200 through libarcllm_cuda.so.
#pragma once
#include <cstdint>
#include <string>
#include <vector>

namespace arcllm::v1::runtime {

enum class EvidenceProfile : std::uint8_t {
    PROFILE_0 = 0,
    PROFILE_1 = 1
};

struct RunRequest {
    std::string model_path;
    // Kept for source compatibility with the Vulkan runtime (its SPIR-V
    // directory); any non-empty value is accepted and otherwise unused.
    std::string shader_dir;
    std::string sidecar_path;
    std::vector<std::uint32_t> input_token_ids;
    std::uint32_t max_new_tokens = 1;
    EvidenceProfile evidence_profile = EvidenceProfile::PROFILE_0;
    bool request_within_validated_domain = false;
};

struct RuntimeStats {
    std::uint32_t prefill_dispatches = 0;       // kernel launches for the prompt
    std::uint32_t prefill_submits = 0;          // CUDA-graph launches for the prompt
    std::uint32_t decode_dispatches_per_step = 0;
    std::uint32_t decode_submits_per_step = 0;
    std::uint32_t decode_steps = 0;

    std::uint32_t route_a_steps = 0;
    std::uint32_t route_b_steps = 0;
    std::uint32_t acquire_events = 0;
    std::uint32_t evict_events = 0;

    std::uint64_t b_allocations = 0;
    std::uint64_t b_materializations = 0;
    std::uint64_t b_validations = 0;
    std::uint64_t b_releases = 0;
    std::uint64_t p1_calls = 0;
    std::uint64_t p3_calls = 0;
    std::uint64_t p0_calls = 0;

    bool finite = false;
};

struct RunResult {
    std::vector<std::uint32_t> generated_token_ids;
    RuntimeStats stats{};
};

// Greedy generation for one request (request-scoped: the model is loaded,
// run and released inside the call).  Throws std::runtime_error on any
// violation, as the reference does.
RunResult generate(const RunRequest& request);

}  // namespace arcllm::v1::runtime
