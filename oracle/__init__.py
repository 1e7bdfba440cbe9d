"""ctypes/numpy front end for the oracle libraries (TEST INFRASTRUCTURE ONLY).

Imported by tests/, ``__graft_entry__.smoke()`` and the cpu_baseline leg of
bench.py -- never by the product package ``arcllm_b200``.

``orc`` wraps oracle/lib/liborc.so (the C restatement, built on demand with
gcc); ``ref`` wraps oracle/_ref/libref_cpu.so (the reference's own CPU code)
and is ``None`` wherever that library was not built.
"""
import ctypes as C
import os

import numpy as np

from . import build as _build

_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_vp = C.c_void_p


def _fp(a):
    """float pointer or NULL for None"""
    return None if a is None else a.ctypes.data_as(_vp)


def _load_orc():
    lib = C.CDLL(_build.build_orc())
    sig = {
        "orc_half_to_float": (C.c_float, [C.c_uint16]),
        "orc_float_to_half_rne": (C.c_uint16, [C.c_float]),
        "orc_q4k_dequant_row": (None, [_u8p, _f32p, C.c_uint32]),
        "orc_q6k_dequant_row": (None, [_u8p, _f32p, C.c_uint32]),
        "orc_q4k_dot_row": (C.c_float, [_u8p, _f32p, C.c_uint32]),
        "orc_q6k_dot_row": (C.c_float, [_u8p, _f32p, C.c_uint32]),
        "orc_matmul_q4": (None, [_u8p, C.c_uint32, C.c_uint32, C.c_uint32, _f32p, _vp, _f32p, C.c_int]),
        "orc_matmul_q6": (None, [_u8p, C.c_uint32, C.c_uint32, C.c_uint32, _f32p, _vp, _f32p, C.c_int]),
        "orc_rmsnorm": (None, [_f32p, _f32p, C.c_uint32, C.c_uint32, C.c_float, _f32p]),
        "orc_rope": (None, [_f32p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_float]),
        "orc_swiglu": (None, [_f32p, _f32p, C.c_uint32, _f32p]),
        "orc_add": (None, [_f32p, _f32p, C.c_uint32, _f32p]),
        "orc_attention_cache": (None, [_f32p, _f32p, _f32p] + [C.c_uint32] * 6 + [_f32p]),
        "orc_argmax": (C.c_uint32, [_f32p, C.c_uint32, C.POINTER(C.c_int)]),
        "orc_splitmix64_at": (C.c_uint64, [C.c_uint64, C.c_uint64]),
        "orc_fill_q4k": (None, [_u8p, C.c_uint64, C.c_uint64, C.c_uint64]),
        "orc_fill_q6k": (None, [_u8p, C.c_uint64, C.c_uint64, C.c_uint64]),
        "orc_fill_normal_f32": (None, [_f32p, C.c_uint64, C.c_uint64, C.c_uint64, C.c_float, C.c_float]),
        "orc_fill_normal_f16": (None, [_u16p, C.c_uint64, C.c_uint64, C.c_uint64, C.c_float, C.c_float]),
        "orc_fill_tokens": (None, [_u32p, C.c_uint64, C.c_uint64, C.c_uint32]),
    }
    for name, (res, args) in sig.items():
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    return lib


def _load_ref():
    path = _build.REF_SO
    if not os.path.exists(path):
        try:
            path = _build.build_ref()
        except RuntimeError:
            path = None
    if not path or not os.path.exists(path):
        return None
    lib = C.CDLL(path)
    sig = {
        "ref_half_to_float": (C.c_float, [C.c_uint16]),
        "ref_q4k_dequant_row": (None, [_u8p, _f32p, C.c_uint32]),
        "ref_q6k_dequant_row": (None, [_u8p, _f32p, C.c_uint32]),
        "ref_q4k_dot_row": (C.c_float, [_u8p, _f32p, C.c_uint32]),
        "ref_q6k_dot_row": (C.c_float, [_u8p, _f32p, C.c_uint32]),
        "ref_matmul_q4": (None, [_u8p, C.c_uint32, C.c_uint32, C.c_uint32, _f32p, _vp, _f32p]),
        "ref_matmul_q6": (None, [_u8p, C.c_uint32, C.c_uint32, C.c_uint32, _f32p, _vp, _f32p]),
        "ref_rmsnorm": (None, [_f32p, _f32p, C.c_uint32, C.c_uint32, C.c_float, _f32p]),
        "ref_rope": (None, [_f32p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_float]),
        "ref_swiglu": (None, [_f32p, _f32p, C.c_uint32, _f32p]),
        "ref_add": (None, [_f32p, _f32p, C.c_uint32, _f32p]),
        "ref_attention_cache": (None, [_f32p, _f32p, _f32p, C.c_uint64] + [C.c_uint32] * 6 + [_f32p]),
        "ref_argmax": (C.c_uint32, [_f32p, C.c_uint32, C.POINTER(C.c_int)]),
        "ref_q6cb_decode_value": (C.c_float, [_u8p, C.c_uint32, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
        "ref_q6cb_fixture": (C.c_int, [C.c_uint32, C.c_uint32, C.c_uint64, C.c_int, _u8p, _f32p]),
        "ref_exec148_materialize_block": (None, [_u8p, _u8p]),
        "ref_exec148_source_tuple": (None, [_u8p, _u8p]),
        "ref_sha256": (None, [_u8p, C.c_uint64, _u8p]),
    }
    for name, (res, args) in sig.items():
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    return lib


orc = _load_orc()
ref = _load_ref()

Q4_BLOCK, Q6_BLOCK = 144, 210


def row_bytes(fmt, k):
    return (k // 256) * (Q4_BLOCK if fmt == "q4k" else Q6_BLOCK)


# ---- numpy conveniences over the C restatement ---------------------------
def fill_q4k(rows, k, seed, row_begin=0):
    nb = k // 256
    out = np.empty(rows * nb * Q4_BLOCK, np.uint8)
    orc.orc_fill_q4k(out, row_begin * nb, rows * nb, seed)
    return out


def fill_q6k(rows, k, seed, row_begin=0):
    nb = k // 256
    out = np.empty(rows * nb * Q6_BLOCK, np.uint8)
    orc.orc_fill_q6k(out, row_begin * nb, rows * nb, seed)
    return out


def fill_weights(fmt, rows, k, seed, row_begin=0):
    return (fill_q4k if fmt == "q4k" else fill_q6k)(rows, k, seed, row_begin)


def normal_f32(n, seed, mu=0.0, sigma=1.0, begin=0):
    out = np.empty(n, np.float32)
    orc.orc_fill_normal_f32(out, begin, n, seed, mu, sigma)
    return out


def normal_f16(n, seed, mu=0.0, sigma=1.0, begin=0):
    out = np.empty(n, np.uint16)
    orc.orc_fill_normal_f16(out, begin, n, seed, mu, sigma)
    return out


def tokens(n, seed, vocab):
    out = np.empty(n, np.uint32)
    orc.orc_fill_tokens(out, n, seed, vocab)
    return out


def dequant(fmt, w, rows, k):
    y = np.empty(rows * k, np.float32)
    rb = row_bytes(fmt, k)
    fn = orc.orc_q4k_dequant_row if fmt == "q4k" else orc.orc_q6k_dequant_row
    for r in range(rows):
        fn(w[r * rb:(r + 1) * rb], y[r * k:(r + 1) * k], k)
    return y.reshape(rows, k)


def matvec(fmt, w, rows, k, x, bias=None, threads=1):
    y = np.empty(rows, np.float32)
    fn = orc.orc_matmul_q4 if fmt == "q4k" else orc.orc_matmul_q6
    fn(w, k, rows, 1, np.ascontiguousarray(x, np.float32), _fp(bias), y, threads)
    return y


def rmsnorm(x, gamma, eps):
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    n = gamma.shape[0]
    orc.orc_rmsnorm(x, np.ascontiguousarray(gamma, np.float32), x.size // n, n, eps, y)
    return y


def rope(x, heads, dim, pos_base, theta):
    x = np.array(x, np.float32, copy=True)
    orc.orc_rope(x, x.size // (heads * dim), heads, dim, pos_base, theta)
    return x


def swiglu(g, u):
    y = np.empty_like(g)
    orc.orc_swiglu(g, u, g.size, y)
    return y


def add(a, b):
    y = np.empty_like(a)
    orc.orc_add(a, b, a.size, y)
    return y


def attention_cache(q, kc, vc, layer, pos, max_ctx, q_heads, kv_heads, dim):
    out = np.empty(q_heads * dim, np.float32)
    orc.orc_attention_cache(np.ascontiguousarray(q, np.float32), kc, vc, layer, pos, max_ctx,
                            q_heads, kv_heads, dim, out)
    return out


def argmax(p):
    fin = C.c_int(0)
    i = orc.orc_argmax(np.ascontiguousarray(p, np.float32), p.size, C.byref(fin))
    return int(i), bool(fin.value)


def half_to_float(h):
    return orc.orc_half_to_float(int(h))


def parity_bounds(w_deq_rows, x):
    """The matvec tolerance: max|err| <= 1e-4 * ||x||_2 * max_r max|w_r| and
    rel-L2 <= 1e-3.  Returns the max-abs bound."""
    return 1e-4 * float(np.linalg.norm(x.astype(np.float64))) * float(np.abs(w_deq_rows).max())
