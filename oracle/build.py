"""Build recipe for the oracle (TEST INFRASTRUCTURE ONLY).

Three libraries and one test program:

* ``oracle/lib/liborc.so`` -- the C restatement in ``oracle/orc.c``.  It needs
  only gcc and is rebuilt wherever it is missing (also on a GPU box).
* ``oracle/_ref/libref_policy.so`` -- the reference's OWN policy engine and
  Q4 FFN-down registration (``oracle/ref_policy.cpp``), same conditions.
* ``oracle/_ref/q4_backend_ref_binding`` -- tests/cpp/q4_backend_ref_binding.cpp
  linked with the reference's OWN policy engine, registry, backend binding and
  Q4 FFN-down registration (compiled in place) and libarcllm_runtime.so.
* ``oracle/_ref/libref_cpu.so`` -- the reference's OWN CPU code, compiled in
  place from an ArcLLM checkout (``--reference``, ``ARCLLM_REFERENCE_DIR``, or
  a ``reference`` directory beside this repository)
  through ``oracle/ref_wrap.cpp``.  Nothing is copied out of the reference
  tree.  Built only where that checkout exists; the golden fixtures under
  ``tests/golden/`` carry its outputs elsewhere.

Both use ``-ffp-contract=off`` so fp32 expressions are rounded op by op, as
the reference's arithmetic is.
"""
import argparse
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ORC_SO = os.path.join(HERE, "lib", "liborc.so")
REF_SO = os.path.join(HERE, "_ref", "libref_cpu.so")
REF_POLICY_SO = os.path.join(HERE, "_ref", "libref_policy.so")


def default_reference():
    """The ArcLLM checkout: ARCLLM_REFERENCE_DIR when set, else a directory
    named ``reference`` beside this repository's root (None when neither
    exists)."""
    d = os.environ.get("ARCLLM_REFERENCE_DIR")
    if d:
        return d
    sibling = os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
    return sibling if os.path.isdir(sibling) else None


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("oracle build failed:\n%s\n%s%s" % (" ".join(cmd), r.stdout, r.stderr))


def build_orc(force=False):
    src = os.path.join(HERE, "orc.c")
    if not force and os.path.exists(ORC_SO) and os.path.getmtime(ORC_SO) >= os.path.getmtime(src):
        return ORC_SO
    os.makedirs(os.path.dirname(ORC_SO), exist_ok=True)
    tmp = ORC_SO + ".tmp%d" % os.getpid()
    _run(["gcc", "-std=c11", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared",
          "-pthread", src, "-o", tmp, "-lm"])
    os.replace(tmp, ORC_SO)
    return ORC_SO


def build_ref(reference=None, force=False):
    """Compile the reference's CPU functions in place; returns the .so path or
    None when no reference checkout is present."""
    reference = reference or default_reference()
    if not reference:
        return None
    src_dir = os.path.join(reference, "src")
    if not os.path.isfile(os.path.join(src_dir, "p8c_segmented_access_correctness.cpp")):
        return None
    wrap = os.path.join(HERE, "ref_wrap.cpp")
    if not force and os.path.exists(REF_SO) and os.path.getmtime(REF_SO) >= os.path.getmtime(wrap):
        return REF_SO
    os.makedirs(os.path.dirname(REF_SO), exist_ok=True)
    tmp = REF_SO + ".tmp%d" % os.getpid()
    _run(["g++", "-std=c++17", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared",
          "-w", "-I", os.path.join(HERE, "ref_shim"), "-I", src_dir, wrap, "-o", tmp])
    os.replace(tmp, REF_SO)
    return REF_SO


def build_ref_policy(reference=None, force=False):
    """Compile the reference's generic policy engine (v4), primitive registry
    (v2) and the Q4 FFN-down registration in place through
    oracle/ref_policy.cpp; returns the .so path or None without a checkout."""
    reference = reference or default_reference()
    if not reference:
        return None
    src_dir = os.path.join(reference, "src")
    if not os.path.isfile(os.path.join(src_dir, "arcllm_v1_generic_policy_engine_v4.cpp")):
        return None
    wrap = os.path.join(HERE, "ref_policy.cpp")
    if not force and os.path.exists(REF_POLICY_SO) and os.path.getmtime(REF_POLICY_SO) >= os.path.getmtime(wrap):
        return REF_POLICY_SO
    os.makedirs(os.path.dirname(REF_POLICY_SO), exist_ok=True)
    tmp = REF_POLICY_SO + ".tmp%d" % os.getpid()
    _run(["g++", "-std=c++17", "-O2", "-fPIC", "-shared", "-w", "-I", src_dir, wrap, "-o", tmp])
    os.replace(tmp, REF_POLICY_SO)
    return REF_POLICY_SO


def build_ref_binding(reference=None, force=False):
    """Link tests/cpp/q4_backend_ref_binding.cpp -- the CUDA Q4 backend driven
    through scenarios S1-S9 by the reference's own policy engine, registry,
    backend binding and Q4 FFN-down registration, compiled in place from the
    checkout -- into oracle/_ref/q4_backend_ref_binding (it finds
    libarcllm_runtime.so / libarcllm_cuda.so through a relative rpath, so it
    also runs where the checkout is absent).  None without a checkout or
    before the runtime library is built."""
    reference = reference or default_reference()
    if not reference:
        return None
    src_dir = os.path.join(reference, "src")
    ref_srcs = [os.path.join(src_dir, f) for f in (
        "arcllm_v1_generic_policy_engine_v4.cpp", "arcllm_v1_primitive_registry_v2.cpp",
        "arcllm_v1_generic_backend_binding_v4.cpp",
        os.path.join("registrations", "arcllm_v1_q4k_down_reference_registration_v2.cpp"))]
    root = os.path.dirname(HERE)
    pkg = os.path.join(root, "arcllm_b200")
    prog = os.path.join(root, "tests", "cpp", "q4_backend_ref_binding.cpp")
    if not all(os.path.isfile(f) for f in ref_srcs) or not os.path.exists(os.path.join(pkg, "libarcllm_runtime.so")):
        return None
    exe = os.path.join(HERE, "_ref", "q4_backend_ref_binding")
    deps = [prog, os.path.join(root, "include", "arcllm", "v1", "q4_cuda_backend.h"),
            os.path.join(pkg, "libarcllm_runtime.so")]
    if not force and os.path.exists(exe) and all(os.path.getmtime(exe) >= os.path.getmtime(d) for d in deps):
        return exe
    os.makedirs(os.path.dirname(exe), exist_ok=True)
    tmp = exe + ".tmp%d" % os.getpid()
    _run(["g++", "-std=c++17", "-O1", "-w", "-DARCLLM_BINDING_FROM_REFERENCE", "-I", os.path.join(root, "include"),
          "-I", os.path.join(reference, "include"), "-I", src_dir, prog] + ref_srcs +
         ["-o", tmp, "-L", pkg, "-larcllm_runtime", "-larcllm_cuda", "-Wl,-rpath,$ORIGIN/../../arcllm_b200"])
    os.replace(tmp, exe)
    return exe


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None)
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args(argv)
    print("orc:", build_orc(a.force))
    print("ref:", build_ref(a.reference, a.force))
    print("ref policy:", build_ref_policy(a.reference, a.force))
    print("ref binding:", build_ref_binding(a.reference, a.force))


if __name__ == "__main__":
    sys.exit(main())
