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
    st = L.arcllm_cuda_stream_delay_us(1000001, None)
    assert L.arcllm_cuda_status_string(st) == b"ARC_E_INVALID_ARGUMENT"


def test_allgather_layout_and_argument_validation():
    """Exchange-buffer layout and the all-gather matvec's argument checks
    (all before any device work)."""
    L = A.lib()
    name = L.arcllm_cuda_status_string
    n = C.c_uint64(0)
    off = C.c_uint64(0)
    # 64-bit epoch-tagged words of every row, then the fp32 logits at a 256-byte boundary
    assert L.arcllm_cuda_allgather_buffer_bytes(6016, C.byref(n)) == 0 and n.value == 48128 + 24064
    assert L.arcllm_cuda_allgather_logits_offset(6016, C.byref(off)) == 0 and off.value == 48128
    assert L.arcllm_cuda_allgather_buffer_bytes(6017, C.byref(n)) == 0 and n.value == 48384 + 24320
    assert L.arcllm_cuda_allgather_logits_offset(6017, C.byref(off)) == 0 and off.value == 48384
    assert name(L.arcllm_cuda_allgather_logits_offset(0, C.byref(off))) == b"ARC_E_INVALID_ARGUMENT"
    ag = L.arcllm_cuda_matvec_allgather
    w, x = C.c_void_p(256), C.c_void_p(256)
    ok = (C.c_void_p * 2)(256, 512)
    cases = [
        ((A.GGML_Q6_K, w, 3008, 3584, x, 0, 6016, ok, 0, 0, 1, 0, None), b"ARC_E_INVALID_ARGUMENT"),  # no ranks
        ((A.GGML_Q6_K, w, 3008, 3584, x, 0, 6016, ok, 2, 2, 1, 0, None), b"ARC_E_INVALID_ARGUMENT"),  # rank >= n
        ((A.GGML_Q6_K, w, 3008, 3584, x, 0, 6016, ok, 2, 0, 0, 0, None), b"ARC_E_INVALID_ARGUMENT"),  # epoch 0
        ((A.GGML_Q6_K, w, 3008, 3584, x, 3009, 6016, ok, 2, 1, 1, 0, None), b"ARC_E_INVALID_ARGUMENT"),  # past end
        ((13, w, 3008, 3584, x, 0, 6016, ok, 2, 0, 1, 0, None), b"ARC_E_INVALID_ARGUMENT"),  # type
        ((A.GGML_Q6_K, w, 3008, 4096, x, 0, 6016, ok, 2, 0, 1, 0, None), b"ARC_E_UNSUPPORTED_SHAPE"),  # K
        ((A.GGML_Q6_K, w, 3008, 3584, x, 0, 6016, (C.c_void_p * 2)(256, 100), 2, 0, 1, 0, None),
         b"ARC_E_ALIGNMENT"),
    ]
    for args, want in cases:
        assert name(ag(*args)) == want, args
    # the host-IO form runs the same checks (x_dev in place of x), plus its host pointers, before any device work
    agh = L.arcllm_cuda_matvec_allgather_hostio
    xh, yh = C.c_void_p(4096), C.c_void_p(8192)
    for args, want in cases:
        t, w_, rows, k, xd, row0, total, bufs, n_r, rank, ep, tmo, st = args
        assert name(agh(t, w_, rows, k, xh, xd, row0, total, bufs, n_r, rank, ep, tmo, yh, st)) == want, args
    good = (A.GGML_Q6_K, w, 3008, 3584, xh, x, 0, 6016, ok, 2, 0, 1, 0, yh, None)
    for i in (4, 5, 13):  # null x_host, x_dev, y_host
        bad = list(good)
        bad[i] = None
        assert name(agh(*bad)) == b"ARC_E_INVALID_ARGUMENT", i


def test_shard_rows_cover_and_align():
    """arcllm_cuda_shard_rows (host-only): the tensor-parallel row shards tile
    [0, n) in rank order, in whole aligned units, balanced to one unit."""
    for n, align in ((18944, 32), (3584, 32), (152064, 32), (1024, 32)):
        for world in (1, 2, 3, 4, 8):
            if n // align < world:
                continue
            spans = []
            for r in range(world):
                r0, rows = C.c_uint32(0), C.c_uint32(0)
                A.call("arcllm_cuda_shard_rows", n, align, world, r, C.byref(r0), C.byref(rows))
                spans.append((r0.value, rows.value))
            assert spans[0][0] == 0 and sum(s[1] for s in spans) == n
            assert all(a[0] + a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert all(s[0] % align == 0 and s[1] % align == 0 for s in spans)
            assert max(s[1] for s in spans) - min(s[1] for s in spans) <= align
