"""EXEC148 (primitive B of the Q4 FFN-down capability) on the GPU: the
materialisation must reproduce the reference materializer's bytes exactly
(golden vectors made by src/q4_down_exec148_materializer.h), identity
validation must accept the exact image and reject a single changed code, and
the EXEC148 matvec must meet the matvec tolerance against the CPU oracle."""
import ctypes as C

import numpy as np
import pytest

import arcllm_b200 as A
import oracle as O
import gpu_util as G
from test_matvec_gpu import assert_matvec_close, gpu_fill, max_abs_w, run_matvec

pytestmark = pytest.mark.gpu


def materialize(src_dev, n_blocks):
    img = G.empty_u8(148 * n_blocks + 16)
    A.call("arcllm_cuda_exec148_materialize", G.ptr(src_dev), n_blocks, G.ptr(img), G.stream())
    return img


def validate(src_dev, img, n_blocks):
    mm = C.c_uint64(0)
    A.call("arcllm_cuda_exec148_validate", G.ptr(src_dev), G.ptr(img), n_blocks, C.byref(mm), G.stream())
    return mm.value


def test_materialize_matches_reference_bytes(golden):
    src = golden["exec148_src"]
    n = src.size // 144
    img = materialize(G.to_dev(src), n)
    assert np.array_equal(G.host(img)[:148 * n], golden["exec148_exe"])
    G.check_device_error()


@pytest.mark.parametrize("rows,k", [(64, 18944), (3, 256)])
def test_validate_exact_and_corrupted(rows, k):
    n = rows * (k // 256)
    src = gpu_fill("q4k", rows, k, 31 + rows)
    img = materialize(src, n)
    assert validate(src, img, n) == 0
    bad = img.clone()
    bad[148 * (n // 2) + 20 + 7] ^= 0x10  # one code nibble of one block
    assert validate(src, bad, n) == 1
    bad2 = img.clone()
    bad2[148 * (n - 1) + 5] ^= 1  # a min byte of the last block
    assert validate(src, bad2, n) == 1
    G.check_device_error()


@pytest.mark.parametrize("rows,k,with_res,impl", [(3584, 18944, True, ""), (3584, 18944, True, "cuda"),
                                                  (5000, 3584, False, ""), (64, 2560, True, ""), (2, 18944, False, ""),
                                                  (37, 512, True, ""), (1, 256, False, "")])
def test_exec148_matvec_parity(rows, k, with_res, impl, monkeypatch):
    """Even row counts run on the K-slice integer-MMA kernel (the image read
    in 2-row tensor-map super-rows, codes as element pairs), odd ones and
    ARCLLM_MATVEC_IMPL=cuda on the CUDA-core kernel."""
    if impl:
        monkeypatch.setenv("ARCLLM_MATVEC_IMPL", impl)
    seed = 77 + rows
    src = gpu_fill("q4k", rows, k, seed)
    img = materialize(src, rows * (k // 256))
    x = O.normal_f32(k, seed + 1)
    res = O.normal_f32(rows, seed + 2) if with_res else None
    y = run_matvec_exec(img, rows, k, x, res)
    y_ref = O.matvec("q4k", O.fill_weights("q4k", rows, k, seed), rows, k, x, threads=8)
    if with_res:
        y_ref = O.add(res, y_ref)
    assert_matvec_close(y, y_ref, x, max_abs_w("q4k", src, rows, k), "EXEC148 %dx%d" % (rows, k))
    G.check_device_error()


def run_matvec_exec(img, rows, k, x, res):
    y = G.empty_f32(rows)
    xd = G.to_dev(x)
    rd = G.to_dev(res) if res is not None else None
    A.call("arcllm_cuda_matvec", A.TYPE_EXEC148, G.ptr(img), rows, k, G.ptr(xd), None, C.c_float(0), None,
           G.ptr(rd) if rd is not None else None, G.ptr(y), G.stream())
    return G.host(y)
