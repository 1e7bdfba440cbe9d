"""Generate tests/golden/policy_q4_down.npz from the reference's OWN policy
engine (oracle/_ref/libref_policy.so, built in place by oracle/build.py from
src/arcllm_v1_generic_policy_engine_v4.cpp, src/arcllm_v1_primitive_registry_v2.cpp
and src/registrations/arcllm_v1_q4k_down_reference_registration_v2.cpp).

For every input of the sweep -- profile 0/1, inside/outside the validated
domain, future reuse 0..40 tokens, primitive B resident or not, its identity
valid or not, each of the P1/P3/P0 acquisition paths available or not -- it
records the engine's decision: status, route, lifecycle, acquisition, reason,
threshold units, requested residency bytes, preserve/validate flags.  The
fixture lets tests/test_policy_pin_cpu.py pin the restated policy where the
reference checkout is absent.  Usage:  python tests/golden/make_policy_golden.py
"""
import ctypes as C
import itertools
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))


def sweep_inputs():
    rows = []
    for p1, scope, reuse, res, valid, avail in itertools.product(range(2), range(2), range(41), range(2), range(2),
                                                                  range(8)):
        rows.append((p1, scope, reuse, res, valid, avail & 1, (avail >> 1) & 1, (avail >> 2) & 1))
    return np.array(rows, np.uint64)


def reference_decisions(inputs):
    from oracle import build
    so = build.build_ref_policy()
    if not so:
        raise SystemExit("the reference policy library is not available (needs the ArcLLM checkout)")
    lib = C.CDLL(so)
    f = lib.ref_q4_down_evaluate
    f.restype = C.c_int
    f.argtypes = [C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]
    out = np.zeros((len(inputs), 8), np.uint64)
    for i, row in enumerate(inputs):
        a = np.ascontiguousarray(row, np.uint64)
        o = np.zeros(8, np.uint64)
        st = f(a.ctypes.data_as(C.POINTER(C.c_uint64)), o.ctypes.data_as(C.POINTER(C.c_uint64)))
        if st:
            raise SystemExit("registry rejected the bundle: %d" % st)
        out[i] = o
    return out


def main():
    inputs = sweep_inputs()
    out = reference_decisions(inputs)
    np.savez_compressed(os.path.join(HERE, "policy_q4_down.npz"), inputs=inputs, decisions=out)
    print("wrote %d decisions" % len(inputs))


if __name__ == "__main__":
    main()
