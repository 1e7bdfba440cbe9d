"""Build recipe for libarcllm_cuda.so (sm_100a only) and the C++ host runtime.

Compiles every ``csrc/*.cu`` with nvcc for ``-gencode arch=compute_100a,code=sm_100a``
into objects under ``arcllm_b200/_build/`` and links them into the in-tree
``arcllm_b200/libarcllm_cuda.so``.  The C++17 host runtime (``runtime/*.cpp``:
GGUF reader, tensor store, Q4CudaBackend, ``arcllm::v1::runtime::generate``) is
compiled with g++ into ``arcllm_b200/libarcllm_runtime.so`` linked against the
CUDA library, plus the ``arcllm_b200/arcllm_v1_runtime_cli`` executable.
Everything is rebuilt only when a source or header is newer.  nvcc
cross-compiles, so this runs without a GPU.
"""
import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OUT = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libarcllm_cuda.so")
RT_SRC = os.path.join(PKG, "runtime")
RT_LIB = os.path.join(PKG, "libarcllm_runtime.so")
RT_CLI = os.path.join(PKG, "arcllm_v1_runtime_cli")
CXX = os.environ.get("CXX", "g++")
CXXFLAGS = ["-std=c++17", "-O2", "-fPIC", "-Wall", "-Wextra", "-I", os.path.join(ROOT, "include")]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include"), "-I", CSRC]


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def _headers():
    return (glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) +
            glob.glob(os.path.join(ROOT, "include", "*.h")))


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("command failed:\n%s\n%s%s" % (" ".join(cmd), r.stdout, r.stderr))
    return r.stdout + r.stderr


def build(force=False, verbose_ptxas=False, jobs=None):
    os.makedirs(OUT, exist_ok=True)
    hdr_mtime = max([os.path.getmtime(h) for h in _headers()] + [os.path.getmtime(__file__)])
    objs, todo = [], []
    for src in _sources():
        obj = os.path.join(OUT, os.path.basename(src) + ".o")
        objs.append(obj)
        if force or not os.path.exists(obj) or os.path.getmtime(obj) < max(os.path.getmtime(src), hdr_mtime):
            todo.append((src, obj))
    logs = []

    def compile_one(so):
        src, obj = so
        cmd = [NVCC] + ARCH + FLAGS + (["-Xptxas", "-v"] if verbose_ptxas else []) + ["-c", src, "-o", obj + ".tmp"]
        out = _run(cmd)
        os.replace(obj + ".tmp", obj)
        return out

    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(8, len(todo))) as ex:
            logs = list(ex.map(compile_one, todo))
    if todo or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        tmp = LIB + ".tmp%d" % os.getpid()
        _run([NVCC] + ARCH + ["-shared", "-Xcompiler", "-fPIC", "-o", tmp] + objs + ["-lcuda"])
        os.replace(tmp, LIB)
    return LIB, logs


def _stale(target, deps):
    return not os.path.exists(target) or os.path.getmtime(target) < max(os.path.getmtime(d) for d in deps)


def build_runtime(force=False):
    """g++ the host runtime into libarcllm_runtime.so (+ the CLI), linked to libarcllm_cuda.so."""
    srcs = sorted(s for s in glob.glob(os.path.join(RT_SRC, "*.cpp")) if not s.endswith("_cli.cpp"))
    hdrs = glob.glob(os.path.join(ROOT, "include", "*.h")) + glob.glob(os.path.join(ROOT, "include", "arcllm", "v1",
                                                                                    "*.h"))
    deps = srcs + hdrs + [LIB, __file__]
    if force or _stale(RT_LIB, deps):
        tmp = RT_LIB + ".tmp%d" % os.getpid()
        _run([CXX] + CXXFLAGS + ["-shared", "-o", tmp] + srcs +
             ["-L", PKG, "-larcllm_cuda", "-Wl,-rpath,$ORIGIN"])
        os.replace(tmp, RT_LIB)
    cli = os.path.join(RT_SRC, "runtime_cli.cpp")
    if force or _stale(RT_CLI, [cli, RT_LIB] + hdrs):
        tmp = RT_CLI + ".tmp%d" % os.getpid()
        _run([CXX] + CXXFLAGS + ["-o", tmp, cli, "-L", PKG, "-larcllm_runtime", "-larcllm_cuda",
                                 "-Wl,-rpath,$ORIGIN"])
        os.replace(tmp, RT_CLI)
    return RT_LIB, RT_CLI


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true")
    a = ap.parse_args(argv)
    lib, logs = build(a.force, a.ptxas_v)
    for l in logs:
        if l.strip():
            print(l)
    print(lib)
    print(*build_runtime(a.force))


if __name__ == "__main__":
    sys.exit(main())
