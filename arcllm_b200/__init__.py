"""ArcLLM-B200: B200-native (sm_100a) kernels for ArcLLM's decode hot path.

The product is ``libarcllm_cuda.so`` (C ABI, ``include/arcllm_cuda.h``) and the
C++17 runtime built on it.  This module loads that library with ctypes and
exposes it to Python callers (the tests and bench.py).  There is no fallback:
if the library cannot be loaded the import of :func:`lib` raises.
"""
import ctypes as C
import os
import threading

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libarcllm_cuda.so")

GGML_F32, GGML_F16, GGML_Q4_K, GGML_Q6_K = 0, 1, 12, 14
Q4K_BLOCK_BYTES, Q6K_BLOCK_BYTES = 144, 210

_lock = threading.Lock()
_lib = None

_vp, _u32, _u64, _f32, _i32 = C.c_void_p, C.c_uint32, C.c_uint64, C.c_float, C.c_int

# name -> argtypes (all return int status unless listed in _RESTYPE)
SIGNATURES = {
    "arcllm_cuda_abi_version": [],
    "arcllm_cuda_status_string": [_i32],
    "arcllm_cuda_last_error_message": [],
    "arcllm_cuda_device_error": [_vp, C.POINTER(_u32)],
    "arcllm_cuda_dequant_q4k": [_vp, _u64, _vp, _vp],
    "arcllm_cuda_dequant_q6k": [_vp, _u64, _vp, _vp],
    "arcllm_cuda_matvec": [_i32, _vp, _u32, _u32, _vp, _vp, _f32, _vp, _vp, _vp, _vp],
    "arcllm_cuda_matvec_hostio": [_i32, _vp, _u32, _u32, _vp, _vp, _vp, _vp, _vp],
    "arcllm_cuda_matvec_q4k": [_vp, _u32, _u32, _vp, _vp, _vp, _vp],
    "arcllm_cuda_matvec_q6k": [_vp, _u32, _u32, _vp, _vp, _vp, _vp],
    "arcllm_cuda_gateup_silu_q4k": [_vp, _vp, _u32, _u32, _vp, _vp, _f32, _vp, _vp],
    "arcllm_cuda_fill_q4k": [_vp, _u64, _u64, _u64, _vp],
    "arcllm_cuda_fill_q6k": [_vp, _u64, _u64, _u64, _vp],
    "arcllm_cuda_fill_normal_f32": [_vp, _u64, _u64, _u64, _f32, _f32, _vp],
    "arcllm_cuda_fill_normal_f16": [_vp, _u64, _u64, _u64, _f32, _f32, _vp],
}
_RESTYPE = {
    "arcllm_cuda_status_string": C.c_char_p,
    "arcllm_cuda_last_error_message": C.c_char_p,
}


class ArcError(RuntimeError):
    def __init__(self, status, message):
        super().__init__("%s: %s" % (status, message))
        self.status = status


def compile_library(force=False):
    """Compile the CUDA library in-tree (nvcc, sm_100a)."""
    import importlib
    return importlib.import_module(__name__ + ".build").build(force=force)[0]


def lib():
    """The loaded libarcllm_cuda.so (built on first use if absent)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                compile_library()
            L = C.CDLL(LIB_PATH)
            for name, args in SIGNATURES.items():
                f = getattr(L, name)
                f.argtypes = args
                f.restype = _RESTYPE.get(name, C.c_int)
            _lib = L
    return _lib


def check(status, what=""):
    if status != 0:
        L = lib()
        msg = L.arcllm_cuda_last_error_message().decode(errors="replace")
        name = L.arcllm_cuda_status_string(status).decode()
        raise ArcError(name, (what + ": " if what else "") + msg)
    return status


def call(name, *args):
    """Invoke an entry point and raise ArcError on a non-zero status."""
    return check(getattr(lib(), name)(*args), name)


def row_bytes(ggml_type, k):
    return (k // 256) * (Q4K_BLOCK_BYTES if ggml_type == GGML_Q4_K else Q6K_BLOCK_BYTES)
