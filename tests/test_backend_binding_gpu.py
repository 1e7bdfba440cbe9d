"""Q4CudaBackend plugged into the reference's OWN policy layer: the program
oracle/_ref/q4_backend_ref_binding (tests/cpp/q4_backend_ref_binding.cpp,
built by oracle/build.py against the reference's headers and linked with its
policy engine, registry, backend binding and Q4 FFN-down registration sources)
replays scenarios S1-S9 of the reference's Vulkan backend validation
(src/arcllm_v1_q4_vulkan_backend_v4.cpp:661-841): A without any B
acquisition, no hidden retry when P1 is unavailable, P1 acquire + identity
validation + route B, resident-B reuse, eviction at zero reuse, P0 and P3
chosen by the policy, final evictions -- every decision from
policy_v4::evaluate, carried out by binding_v4::apply_decision on the CUDA
backend, every routed primitive executed and compared with the plain Q4_K
matvec (rel-L2 1e-5); plus a corrupted P3 sidecar that fails validation and
is released.  The program is prebuilt where the ArcLLM checkout is present
and travels with the repository; the test is skipped where it was never
built."""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXE = os.path.join(ROOT, "oracle", "_ref", "q4_backend_ref_binding")


def test_q4_backend_scenarios_through_reference_policy_layer(tmp_path):
    if not os.path.exists(EXE):
        pytest.skip("oracle/_ref/q4_backend_ref_binding was not built (needs the ArcLLM checkout)")
    r = subprocess.run([EXE, str(tmp_path)], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failure(s)" in r.stdout
