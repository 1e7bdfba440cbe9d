"""Build recipe for libarcllm_cuda.so (sm_100a only).

Compiles every ``csrc/*.cu`` with nvcc for ``-gencode arch=compute_100a,code=sm_100a``
into objects under ``arcllm_b200/_build/`` and links them into the in-tree
``arcllm_b200/libarcllm_cuda.so``.  The objects are rebuilt only when a
source or header is newer.  nvcc cross-compiles, so this runs without a GPU.
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


if __name__ == "__main__":
    sys.exit(main())
