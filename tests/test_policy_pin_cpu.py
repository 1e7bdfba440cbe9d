"""The restated Q4 FFN-down route selection (decide_q4_down,
arcllm_b200/runtime/q4_down_policy.cpp) against the reference's OWN generic
policy engine (src/arcllm_v1_generic_policy_engine_v4.cpp:103-317 evaluating
the bundle of src/registrations/arcllm_v1_q4k_down_reference_registration_v2.cpp),
decision for decision over 5248 inputs: profile 0/1 x inside/outside the
validated domain x future reuse 0..40 x B resident x B identity valid x the
P1/P3/P0 acquisition paths available or not, under generate()'s runtime
conditions (model loaded, acquisition allowed, primitives executable, lease
granted).  Every field is compared: route, lifecycle action, acquisition
path, reason, threshold units, requested residency bytes, the preserve and
validate flags; the engine's status must be OK throughout (the fallback A is
always routable).

The reference side comes from tests/golden/policy_q4_down.npz (written by
tests/golden/make_policy_golden.py from the reference library) and, where the
ArcLLM checkout is present, from the live library as well.
"""
import ctypes as C
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "arcllm_b200")
GOLDEN = os.path.join(ROOT, "tests", "golden", "policy_q4_down.npz")


def ours(tmp_path):
    exe = str(tmp_path / "q4_down_policy_sweep")
    src = os.path.join(ROOT, "tests", "cpp", "q4_down_policy_sweep.cpp")
    subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-I", os.path.join(ROOT, "include"), src, "-o", exe,
                    "-L", PKG, "-larcllm_runtime", "-larcllm_cuda", "-Wl,-rpath," + PKG], check=True)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=60, check=True)
    ins, outs = [], []
    for line in r.stdout.splitlines():
        a, b = line.split(":")
        ins.append([int(v) for v in a.split()])
        outs.append([int(v) for v in b.split()])
    return np.array(ins, np.uint64), np.array(outs, np.uint64)


def compare(inputs, decisions, our_in, our_out):
    assert np.array_equal(inputs, our_in), "sweep inputs differ from the golden sweep"
    assert (decisions[:, 0] == 0).all(), "the reference engine returned a non-OK status"
    bad = np.nonzero((decisions[:, 1:] != our_out).any(axis=1))[0]
    msg = "; ".join("in %s: ref %s ours %s" % (inputs[i].tolist(), decisions[i, 1:].tolist(), our_out[i].tolist())
                    for i in bad[:5])
    assert bad.size == 0, "%d of %d decisions differ: %s" % (bad.size, len(inputs), msg)


def test_policy_matches_reference_golden(tmp_path):
    g = np.load(GOLDEN)
    our_in, our_out = ours(tmp_path)
    compare(g["inputs"], g["decisions"], our_in, our_out)
    # the sweep reaches every outcome the policy has under these conditions
    assert set(np.unique(g["decisions"][:, 4]).tolist()) >= {1, 3, 6, 7, 10, 11, 12}


def test_policy_matches_live_reference_engine(tmp_path):
    import sys
    sys.path.insert(0, ROOT)
    from oracle import build
    if not build.build_ref_policy():
        pytest.skip("no ArcLLM checkout to build the reference policy engine from")
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import make_policy_golden as M
    inputs = M.sweep_inputs()
    our_in, our_out = ours(tmp_path)
    compare(inputs, M.reference_decisions(inputs), our_in, our_out)
