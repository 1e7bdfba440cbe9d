"""CPU-only checks of the C-ABI boundary: the library loads, exports every
entry point declared in include/*.h, and rejects bad arguments on the host
before any device work."""
import ctypes as C
import glob
import os
import re
import subprocess

import arcllm_b200 as A

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        txt = open(h).read()
        names.update(re.findall(r"ARCLLM_CUDA_API\s+[\w\s\*]+?\b(arcllm_cuda_\w+)\s*\(", txt))
    return names


def exported_symbols(path):
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True, check=True).stdout
    return {l.split()[-1] for l in out.splitlines() if " T " in l}


def test_library_exports_every_declared_symbol():
    lib = A.lib()
    decl = declared_symbols()
    assert len(decl) >= 14
    exp = exported_symbols(A.LIB_PATH)
    missing = sorted(decl - exp)
    assert not missing, "declared but not exported: %s" % missing
    for name in decl:
        assert hasattr(lib, name)


def test_python_signatures_cover_the_header():
    assert declared_symbols() <= set(A.SIGNATURES)


def test_abi_version_and_status_strings():
    L = A.lib()
    assert L.arcllm_cuda_abi_version() == 1
    assert L.arcllm_cuda_status_string(0) == b"ARC_OK"
    assert L.arcllm_cuda_status_string(2) == b"ARC_E_ALIGNMENT"
    assert L.arcllm_cuda_status_string(99) == b"ARC_E_UNKNOWN"


def test_host_side_argument_validation():
    """These fail in argument checks, before anything touches a device."""
    L = A.lib()
    f = L.arcllm_cuda_matvec
    st = f(A.GGML_Q4_K, None, 8, 3584, None, None, C.c_float(0), None, None, None, None)
    assert st != 0
    st = f(A.GGML_Q4_K, C.c_void_p(16), 8, 300, C.c_void_p(16), None, C.c_float(0), None, None, C.c_void_p(16), None)
    assert L.arcllm_cuda_status_string(st) == b"ARC_E_INVALID_ARGUMENT"
    assert b"multiple of 256" in L.arcllm_cuda_last_error_message()
    st = f(9, C.c_void_p(16), 8, 512, C.c_void_p(16), None, C.c_float(0), None, None, C.c_void_p(16), None)
    assert L.arcllm_cuda_status_string(st) == b"ARC_E_INVALID_ARGUMENT"
    st = L.arcllm_cuda_gateup_silu_q4k(C.c_void_p(16), C.c_void_p(16), 8, 65536, C.c_void_p(16), None,
                                       C.c_float(0), C.c_void_p(16), None)
    assert L.arcllm_cuda_status_string(st) == b"ARC_E_UNSUPPORTED_SHAPE"
    st = L.arcllm_cuda_dequant_q4k(None, 4, None, None)
    assert L.arcllm_cuda_status_string(st) == b"ARC_E_INVALID_ARGUMENT"
