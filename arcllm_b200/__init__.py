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
TYPE_EXEC148 = 148  # EXEC148 image of a Q4_K matrix (route B of the Q4 FFN-down capability)
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
    "arcllm_cuda_allgather_buffer_bytes": [_u32, C.POINTER(_u64)],
    "arcllm_cuda_allgather_logits_offset": [_u32, C.POINTER(_u64)],
    "arcllm_cuda_matvec_allgather": [_i32, _vp, _u32, _u32, _vp, _u32, _u32, C.POINTER(_vp), _u32, _u32, _u32, _u32,
                                     _vp],
    "arcllm_cuda_matvec_allgather_hostio": [_i32, _vp, _u32, _u32, _vp, _vp, _u32, _u32, C.POINTER(_vp), _u32, _u32,
                                            _u32, _u32, _vp, _vp],
    "arcllm_cuda_ipc_get_handle": [_vp, _vp],
    "arcllm_cuda_ipc_open_handle": [_vp, C.POINTER(_vp)],
    "arcllm_cuda_ipc_close_handle": [_vp],
    "arcllm_cuda_matvec_q4k": [_vp, _u32, _u32, _vp, _vp, _vp, _vp],
    "arcllm_cuda_matvec_q6k": [_vp, _u32, _u32, _vp, _vp, _vp, _vp],
    "arcllm_cuda_gateup_silu_q4k": [_vp, _vp, _u32, _u32, _vp, _vp, _f32, _vp, _vp],
    "arcllm_cuda_ffn_block": [_i32, _vp, _vp, _vp, _u32, _u32, _vp, _vp, _f32, _vp, _vp, _vp, _vp],
    "arcllm_cuda_gemm_q4k_bf16": [_vp, _u32, _u32, _vp, _u32, _vp, _vp],
    "arcllm_cuda_gemm_allgather_buffer_bytes": [_u32, _u32, C.POINTER(_u64)],
    "arcllm_cuda_gemm_bf16_allgather": [_i32, _vp, _u32, _u32, _vp, _u32, _u32, _u32, C.POINTER(_vp), _u32, _u32,
                                        _u32, _u32, _vp],
    "arcllm_cuda_gemm_bf16": [_i32, _vp, _u32, _u32, _vp, _u32, _vp, _vp, _vp],
    "arcllm_cuda_gemm_f16": [_i32, _vp, _u32, _u32, _vp, _u32, _vp, _vp, _vp],
    "arcllm_cuda_gemm_f16x3": [_i32, _vp, _u32, _u32, _vp, _vp, _u32, _vp, _vp, _vp],
    "arcllm_cuda_rmsnorm_rows": [_vp, _vp, _f32, _u32, _u32, _i32, _vp, _vp, _vp],
    "arcllm_cuda_rope_kv_rows": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _u32, _u32, _vp, _vp, _u32, _u32, _u32, _u32, _u32,
                                 _vp],
    "arcllm_cuda_attention_prefill": [_vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _u32, _u32, _vp, _vp],
    "arcllm_cuda_exec148_materialize": [_vp, _u64, _vp, _vp],
    "arcllm_cuda_exec148_validate": [_vp, _vp, _u64, C.POINTER(C.c_uint64), _vp],
    "arcllm_cuda_fill_q4k": [_vp, _u64, _u64, _u64, _vp],
    "arcllm_cuda_fill_q6k": [_vp, _u64, _u64, _u64, _vp],
    "arcllm_cuda_fill_normal_f32": [_vp, _u64, _u64, _u64, _f32, _f32, _vp],
    "arcllm_cuda_fill_normal_f16": [_vp, _u64, _u64, _u64, _f32, _f32, _vp],
    "arcllm_cuda_rope_table": [_vp, _u32, _u32, _f32],
    "arcllm_cuda_rope_kv_store": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _vp],
    "arcllm_cuda_attention_decode": [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _u32, _vp, _vp, _vp],
    "arcllm_cuda_attention_decode_noalloc": [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _u32, _vp, _vp],
    "arcllm_cuda_embed": [_i32, _vp, _vp, _u32, _u32, _vp, _vp],
    "arcllm_cuda_argmax": [_vp, _u32, _vp, C.POINTER(_u32), C.POINTER(_i32), _vp],
    "arcllm_cuda_set_launch_overlap": [_i32],
    "arcllm_cuda_set_device": [_i32],
    "arcllm_cuda_device_count": [C.POINTER(C.c_int)],
    "arcllm_cuda_malloc": [_u64, C.POINTER(_vp)],
    "arcllm_cuda_free": [_vp],
    "arcllm_cuda_memcpy_h2d": [_vp, _vp, _u64, _vp],
    "arcllm_cuda_memcpy_d2h": [_vp, _vp, _u64, _vp],
    "arcllm_cuda_stream_create": [C.POINTER(_vp)],
    "arcllm_cuda_stream_destroy": [_vp],
    "arcllm_cuda_stream_synchronize": [_vp],
    "arcllm_cuda_stream_delay_us": [_u32, _vp],
    "arcllm_cuda_model_create": [_vp, C.POINTER(_vp)],
    "arcllm_cuda_model_destroy": [_vp],
    "arcllm_cuda_model_set_layer": [_vp, _u32, _vp],
    "arcllm_cuda_model_set_endpoints": [_vp, _vp, _i32, _vp, _vp, _i32],
    "arcllm_cuda_model_generate": [_vp, _vp, _u32, _u32, _vp, _vp, _vp],
    "arcllm_cuda_model_begin": [_vp, _vp, _u32, _u32, _vp],
    "arcllm_cuda_model_step": [_vp, _i32, _i32, _vp],
    "arcllm_cuda_model_prefill": [_vp, _vp],
    "arcllm_cuda_model_set_prefill_mode": [_vp, _i32],
    "arcllm_cuda_model_set_prefill_down": [_vp, _u32, _vp, _i32],
    "arcllm_cuda_model_logits": [_vp, C.POINTER(_vp)],
    "arcllm_cuda_model_kv_cache": [_vp, C.POINTER(_vp), C.POINTER(_vp)],
    "arcllm_cuda_model_shard_lm_head": [_vp, _u32, _u32],
    "arcllm_cuda_model_tp_exchange_words": [_vp, _u32, C.POINTER(_u32)],
    "arcllm_cuda_model_set_tensor_parallel": [_vp, _vp, _u32, _u32, _u32],
    "arcllm_cuda_exchange_buffer_bytes": [_u32, C.POINTER(C.c_uint64)],
    "arcllm_cuda_exchange_gather": [_vp, _u32, _u32, _u32, _vp, _u32, _u32, _vp, _u32, _u32, _vp],
    "arcllm_cuda_shard_rows": [_u32, _u32, _u32, _u32, C.POINTER(_u32), C.POINTER(_u32)],
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


class ModelConfig(C.Structure):
    _fields_ = [("n_layers", _u32), ("hidden", _u32), ("n_heads", _u32), ("n_kv_heads", _u32),
                ("head_dim", _u32), ("ffn", _u32), ("vocab", _u32), ("max_ctx", _u32),
                ("rms_eps", _f32), ("rope_theta", _f32)]


class Layer(C.Structure):
    _fields_ = [("attn_norm", _vp), ("wq", _vp), ("bq", _vp), ("type_q", _i32),
                ("wk", _vp), ("bk", _vp), ("type_k", _i32), ("wv", _vp), ("bv", _vp), ("type_v", _i32),
                ("wo", _vp), ("type_o", _i32), ("ffn_norm", _vp), ("w_gate", _vp), ("w_up", _vp),
                ("type_gate_up", _i32), ("w_down", _vp), ("type_down", _i32)]


class GenStats(C.Structure):
    _fields_ = [("prefill_launches", _u32), ("prefill_graph_launches", _u32),
                ("decode_launches_per_step", _u32), ("decode_graph_launches_per_step", _u32),
                ("decode_steps", _u32), ("prefill_ms", _f32), ("decode_ms", _f32), ("finite", _i32)]


def row_bytes(ggml_type, k):
    return (k // 256) * (Q4K_BLOCK_BYTES if ggml_type == GGML_Q4_K else Q6K_BLOCK_BYTES)
