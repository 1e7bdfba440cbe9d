"""GPU parity of the dequant / matvec / gate-up kernels against the CPU oracle.

Bars:
  * dequantised values: bit-exact;
  * matvec: max|y - y_ref| <= 1e-4 * ||x||_2 * max_r max|w_r|  and
    ||y - y_ref||_2 / ||y_ref||_2 <= 1e-3;
  * synthetic fixture streams: byte-identical to the oracle's generators.
"""
import ctypes as C

import numpy as np
import pytest

import arcllm_b200 as A
import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
from tests import gpu_util as G  # noqa: E402

FMT = {"q4k": A.GGML_Q4_K, "q6k": A.GGML_Q6_K}
BS = {"q4k": 144, "q6k": 210}


def gpu_fill(fmt, rows, k, seed, row_begin=0):
    nb = k // 256
    t = G.empty_u8(rows * nb * BS[fmt] + 16)
    A.call("arcllm_cuda_fill_" + fmt, G.ptr(t), row_begin * nb, rows * nb, seed, G.stream())
    return t


def gpu_dequant(fmt, w, n_blocks):
    y = G.empty_f32(n_blocks * 256)
    A.call("arcllm_cuda_dequant_" + fmt, G.ptr(w), n_blocks, G.ptr(y), G.stream())
    return y


def max_abs_w(fmt, w, rows, k):
    """max |w| over the tensor, via the (bit-exact) GPU dequant in chunks"""
    nb = k // 256
    m, chunk = 0.0, max(1, (1 << 24) // k)
    for r0 in range(0, rows, chunk):
        r1 = min(rows, r0 + chunk)
        sub = w[r0 * nb * BS[fmt]:]
        y = gpu_dequant(fmt, sub, (r1 - r0) * nb)
        m = max(m, float(y.abs().max()))
    return m


def assert_matvec_close(y, y_ref, x, wmax, what=""):
    y = np.asarray(y, np.float64)
    y_ref = np.asarray(y_ref, np.float64)
    bound = 1e-4 * float(np.linalg.norm(np.asarray(x, np.float64))) * wmax
    err = np.abs(y - y_ref)
    rel = float(np.linalg.norm(y - y_ref) / max(np.linalg.norm(y_ref), 1e-30))
    assert np.all(np.isfinite(y)), what
    assert err.max() <= bound, "%s: max|err| %.3e > bound %.3e" % (what, err.max(), bound)
    assert rel <= 1e-3, "%s: rel-L2 %.3e" % (what, rel)
    return err.max(), bound, rel


# ---------------------------------------------------------------- fixtures
@pytest.mark.parametrize("fmt", ["q4k", "q6k"])
def test_fill_matches_oracle(fmt):
    rows, k = 37, 512
    w = gpu_fill(fmt, rows, k, 0xFEED, row_begin=5)
    ref = O.fill_weights(fmt, rows, k, 0xFEED, row_begin=5)
    assert np.array_equal(G.host(w)[:ref.size], ref)


def test_fill_normal_matches_oracle():
    n = 100003
    t = G.empty_f32(n)
    A.call("arcllm_cuda_fill_normal_f32", G.ptr(t), 7, n, 0xABC, C.c_float(1.0), C.c_float(0.1), G.stream())
    assert np.array_equal(G.host(t).view(np.uint32), O.normal_f32(n, 0xABC, 1.0, 0.1, begin=7).view(np.uint32))
    h = torch.empty(n, dtype=torch.int16, device=G.dev())
    A.call("arcllm_cuda_fill_normal_f16", G.ptr(h), 0, n, 0xABD, C.c_float(0.0), C.c_float(0.02), G.stream())
    assert np.array_equal(G.host(h).view(np.uint16), O.normal_f16(n, 0xABD, 0.0, 0.02))


# ---------------------------------------------------------------- dequant
@pytest.mark.parametrize("fmt", ["q4k", "q6k"])
def test_dequant_bit_exact_golden(golden, fmt):
    w = golden[fmt + "_deq_w"]
    y = gpu_dequant(fmt, G.to_dev(w), w.size // BS[fmt])
    assert np.array_equal(G.host(y).view(np.uint32), golden[fmt + "_deq_y"].view(np.uint32))


@pytest.mark.parametrize("fmt,rows,k", [("q4k", 256, 3584), ("q6k", 256, 3584), ("q6k", 16, 18944)])
def test_dequant_bit_exact_config(fmt, rows, k):
    w = gpu_fill(fmt, rows, k, 77)
    y = gpu_dequant(fmt, w, rows * (k // 256))
    ref = O.dequant(fmt, O.fill_weights(fmt, rows, k, 77), rows, k).ravel()
    assert np.array_equal(G.host(y).view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("s", range(5))
def test_dequant_q6_strata(golden, s):
    w = golden["q6cb_%d_w" % s]
    y = gpu_dequant("q6k", G.to_dev(w), w.size // 210)
    assert np.array_equal(G.host(y).view(np.uint32), golden["q6cb_%d_deq" % s].view(np.uint32))


# ---------------------------------------------------------------- matvec
def run_matvec(fmt, w, rows, k, x, gamma=None, eps=1e-6, bias=None, residual=None):
    y = G.empty_f32(rows)
    xd = G.to_dev(x)
    gd = None if gamma is None else G.to_dev(gamma)
    bd = None if bias is None else G.to_dev(bias)
    rd = None if residual is None else G.to_dev(residual)
    A.call("arcllm_cuda_matvec", FMT[fmt], G.ptr(w), rows, k, G.ptr(xd), G.ptr(gd), C.c_float(eps), G.ptr(bd),
           G.ptr(rd), G.ptr(y), G.stream())
    return G.host(y)


CASES = [
    # (fmt, rows, k) -- BASELINE shapes plus ragged / tiny edge cases
    ("q4k", 18944, 3584),   # config 0: gate/up shape
    ("q4k", 3584, 18944),   # FFN down, Q4 layers
    ("q4k", 512, 3584),     # K projection
    ("q6k", 152064, 3584),  # config 1: LM head
    ("q6k", 3584, 18944),   # config 1: FFN down
    ("q6k", 512, 3584),     # V projection
    ("q4k", 1, 256),
    ("q6k", 1, 256),        # single row of a single super-block: ragged 210-byte group
    ("q6k", 37, 3584),      # rows not a multiple of the row group
    ("q4k", 37, 512),
    ("q6k", 13, 18944),
    ("q6k", 5, 768),        # odd block count per row
    ("q4k", 1, 18944),
    ("q6k", 2, 4096),
    ("q4k", 40, 4608),
    ("q6k", 700, 18944),
]

# split-K tensor-core kernel (opt-in for K > 3584): single row, several 32-row
# groups, ragged last group, K not a multiple of the 6-super-block chunk, more
# work units than SMs, a 13-row matrix whose last row ends inside a 16-byte word
# Q6_K rows must be a multiple of 4 for the long-K tensor-core kernel; the
# other Q6_K cases check that those shapes fall back to the CUDA-core kernel.
SPLITK_CASES = [("q4k", 1, 18944), ("q6k", 2, 4096), ("q4k", 40, 4608), ("q6k", 700, 18944), ("q6k", 13, 18944),
                ("q4k", 3584, 18944), ("q6k", 3584, 18944), ("q6k", 12, 18944), ("q6k", 4, 4096), ("q4k", 3, 18944),
                ("q4k", 1000, 32768)]


@pytest.mark.parametrize("fmt,rows,k", CASES)
def test_matvec_parity(fmt, rows, k):
    seed = 1000 + rows + k
    w = gpu_fill(fmt, rows, k, seed)
    x = O.normal_f32(k, seed + 1)
    bias = O.normal_f32(rows, seed + 2, 0.0, 0.02)
    y = run_matvec(fmt, w, rows, k, x, bias=bias)
    y_ref = O.matvec(fmt, O.fill_weights(fmt, rows, k, seed), rows, k, x, bias, threads=8)
    assert_matvec_close(y, y_ref, x, max_abs_w(fmt, w, rows, k), "%s %dx%d" % (fmt, rows, k))
    G.check_device_error()


@pytest.mark.parametrize("fmt,rows,k", SPLITK_CASES)
def test_matvec_splitk_parity(fmt, rows, k):
    test_matvec_parity(fmt, rows, k)


# the CUDA-core streaming kernel (ARCLLM_MATVEC_IMPL=cuda) on the shapes the
# tensor-core kernels take by default
@pytest.mark.parametrize("fmt,rows,k", [("q6k", 3584, 18944), ("q4k", 3584, 18944), ("q6k", 700, 3584),
                                        ("q4k", 13, 4608)])
def test_matvec_cuda_core_parity(fmt, rows, k, monkeypatch):
    monkeypatch.setenv("ARCLLM_MATVEC_IMPL", "cuda")
    test_matvec_parity(fmt, rows, k)


@pytest.mark.parametrize("fmt", ["q4k", "q6k"])
def test_matvec_splitk_repeat_bit_identical(fmt):
    """The cross-CTA reduction re-arms its counters and adds slice partials in
    a fixed order: back-to-back launches give bit-identical rows."""
    rows, k, seed = 3584, 18944, 5151
    w = gpu_fill(fmt, rows, k, seed)
    x = O.normal_f32(k, seed + 1)
    ys = [run_matvec(fmt, w, rows, k, x) for _ in range(3)]
    assert np.array_equal(ys[0].view(np.uint32), ys[1].view(np.uint32))
    assert np.array_equal(ys[0].view(np.uint32), ys[2].view(np.uint32))
    G.check_device_error()


@pytest.mark.parametrize("fmt", ["q4k", "q6k"])
def test_matvec_splitk_rmsnorm_residual(fmt):
    rows, k, seed = 200, 18944, 4343
    w = gpu_fill(fmt, rows, k, seed)
    x = O.normal_f32(k, seed + 1)
    gamma = O.normal_f32(k, seed + 2, 1.0, 0.1)
    res = O.normal_f32(rows, seed + 3)
    y = run_matvec(fmt, w, rows, k, x, gamma=gamma, residual=res)
    xn = O.rmsnorm(x, gamma, 1e-6)
    y_ref = O.add(res, O.matvec(fmt, O.fill_weights(fmt, rows, k, seed), rows, k, xn, threads=8))
    assert_matvec_close(y, y_ref, xn, max_abs_w(fmt, w, rows, k), fmt + " split-K rmsnorm+residual")


@pytest.mark.parametrize("fmt", ["q4k", "q6k"])
def test_matvec_rmsnorm_residual(fmt):
    rows, k, seed = 3584, 3584, 4242
    w = gpu_fill(fmt, rows, k, seed)
    x = O.normal_f32(k, seed + 1)
    gamma = O.normal_f32(k, seed + 2, 1.0, 0.1)
    res = O.normal_f32(rows, seed + 3)
    y = run_matvec(fmt, w, rows, k, x, gamma=gamma, residual=res)
    xn = O.rmsnorm(x, gamma, 1e-6)
    y_ref = O.add(res, O.matvec(fmt, O.fill_weights(fmt, rows, k, seed), rows, k, xn, threads=8))
    assert_matvec_close(y, y_ref, xn, max_abs_w(fmt, w, rows, k), fmt + " rmsnorm+residual")


@pytest.mark.parametrize("fmt", ["q4k", "q6k"])
def test_matvec_golden_reference_outputs(golden, fmt):
    """Against the reference's own matmul outputs stored in the golden file."""
    for k in (3584, 18944):
        tag = "%s_mv_%d" % (fmt, k)
        rows, wseed, xseed, bseed = [int(v) for v in golden[tag + "_seeds"]]
        w = gpu_fill(fmt, rows, k, wseed)
        x = O.normal_f32(k, xseed)
        bias = O.normal_f32(rows, bseed, 0.0, 0.02)
        y = run_matvec(fmt, w, rows, k, x, bias=bias)
        assert_matvec_close(y, golden[tag + "_yb"], x, max_abs_w(fmt, w, rows, k), tag)


@pytest.mark.parametrize("s", range(5))
def test_matvec_q6_strata(golden, s):
    """Q6_K conditioning strata, HIGH_CANCELLATION included (different
    summation order than the reference's sequential fp32 loop)."""
    w, x = golden["q6cb_%d_w" % s], golden["q6cb_%d_x" % s]
    n = x.size
    rows = w.size // ((n // 256) * 210)
    wd = G.empty_u8(w.size + 16)
    wd[:w.size].copy_(torch.from_numpy(w))
    y = run_matvec("q6k", wd, rows, n, x)
    wmax = float(np.abs(golden["q6cb_%d_deq" % s]).max())
    assert_matvec_close(y, golden["q6cb_%d_y" % s], x, wmax, "q6cb stratum %d" % s)


@pytest.mark.parametrize("rows,k", [(18944, 3584), (37, 3584), (3, 512)])
def test_gateup_silu(rows, k):
    seed = 555 + rows
    wg = gpu_fill("q4k", rows, k, seed)
    wu = gpu_fill("q4k", rows, k, seed + 1)
    x = O.normal_f32(k, seed + 2)
    gamma = O.normal_f32(k, seed + 3, 1.0, 0.1)
    s = G.empty_f32(rows)
    xd, gd = G.to_dev(x), G.to_dev(gamma)  # keep both alive across the launch
    A.call("arcllm_cuda_gateup_silu_q4k", G.ptr(wg), G.ptr(wu), rows, k, G.ptr(xd), G.ptr(gd), C.c_float(1e-6),
           G.ptr(s), G.stream())
    xn = O.rmsnorm(x, gamma, 1e-6)
    g = O.matvec("q4k", O.fill_q4k(rows, k, seed), rows, k, xn, threads=8)
    u = O.matvec("q4k", O.fill_q4k(rows, k, seed + 1), rows, k, xn, threads=8)
    s_ref = O.swiglu(g, u)
    wmax = max(max_abs_w("q4k", wg, rows, k), max_abs_w("q4k", wu, rows, k))
    b = 1e-4 * float(np.linalg.norm(xn.astype(np.float64))) * wmax
    sil = g / (1 + np.exp(-g.astype(np.float64)))
    bound = 1.2 * (b * float(np.abs(u).max()) + b * float(np.abs(sil).max()) + b * b)
    out = G.host(s).astype(np.float64)
    assert np.abs(out - s_ref).max() <= bound
    assert np.linalg.norm(out - s_ref) / np.linalg.norm(s_ref) <= 1e-3
    G.check_device_error()


def test_matvec_rejects_bad_arguments():
    w = gpu_fill("q6k", 8, 512, 1)
    x = G.to_dev(O.normal_f32(512, 2))
    y = G.empty_f32(8)
    L = A.lib()
    st = L.arcllm_cuda_matvec(A.GGML_Q6_K, C.c_void_p(w.data_ptr() + 2), 8, 512, G.ptr(x), None, C.c_float(0), None,
                              None, G.ptr(y), G.stream())
    assert L.arcllm_cuda_status_string(st) == b"ARC_E_ALIGNMENT"
    st = L.arcllm_cuda_matvec(A.GGML_Q6_K, G.ptr(w), 8, 500, G.ptr(x), None, C.c_float(0), None, None, G.ptr(y),
                              G.stream())
    assert L.arcllm_cuda_status_string(st) == b"ARC_E_INVALID_ARGUMENT"
    st = L.arcllm_cuda_matvec(7, G.ptr(w), 8, 512, G.ptr(x), None, C.c_float(0), None, None, G.ptr(y), G.stream())
    assert L.arcllm_cuda_status_string(st) == b"ARC_E_INVALID_ARGUMENT"


@pytest.mark.parametrize("fmt", ["q4k", "q6k"])
@pytest.mark.parametrize("scale", [1e-30, 1.0, 1e25])
def test_matvec_x_dynamic_range(fmt, scale):
    """Activations far from unit scale, with per-block outliers: the matvec
    must stay within the tolerance relative to ||x|| at any magnitude."""
    rows, k, seed = 96, 3584, 777
    w = gpu_fill(fmt, rows, k, seed)
    x = O.normal_f32(k, seed + 1)
    x[::97] *= 1000.0  # one large value in many 32-element blocks
    x[5:40] = 0.0      # an all-zero block and a partly zero one
    x = (x.astype(np.float64) * scale).astype(np.float32)
    y = run_matvec(fmt, w, rows, k, x)
    y_ref = O.matvec(fmt, O.fill_weights(fmt, rows, k, seed), rows, k, x, threads=8)
    assert_matvec_close(y, y_ref, x, max_abs_w(fmt, w, rows, k), "%s x scale %g" % (fmt, scale))


@pytest.mark.parametrize("fmt", ["q4k", "q6k"])
@pytest.mark.parametrize("bad", [np.nan, np.inf])
def test_matvec_nonfinite_x_propagates(fmt, bad):
    """A non-finite activation makes every output non-finite, as the
    reference's fp32 loop does (the runtime then refuses the logits)."""
    rows, k, seed = 40, 3584, 778
    w = gpu_fill(fmt, rows, k, seed)
    x = O.normal_f32(k, seed + 1)
    x[1234] = bad
    y = run_matvec(fmt, w, rows, k, x)
    y_ref = O.matvec(fmt, O.fill_weights(fmt, rows, k, seed), rows, k, x, threads=8)
    assert not np.isfinite(y_ref).any()
    assert not np.isfinite(y).any()
    G.check_device_error()


@pytest.mark.parametrize("pinned", [True, False])
@pytest.mark.parametrize("fmt,rows,k", [("q6k", 152064 // 8, 3584), ("q4k", 3584, 18944)])
def test_matvec_hostio_pinned_and_pageable(pinned, fmt, rows, k):
    """arcllm_cuda_matvec_hostio: a pinned y_host is written by the kernel
    itself (mapped host memory), a pageable one by a copy afterwards.  Whole-row
    (LM-head shard) and K-slice (FFN down) kernels; three calls with a different
    x each hold the device matvec's rows bit for bit."""
    seed = 3131
    w = gpu_fill(fmt, rows, k, seed)
    xd, yd = G.empty_f32(k), G.empty_f32(rows)
    xh = torch.empty(k, dtype=torch.float32)
    yh = torch.full((rows,), float("nan"), dtype=torch.float32)
    if pinned:
        xh, yh = xh.pin_memory(), yh.pin_memory()
    ty = A.GGML_Q6_K if fmt == "q6k" else A.GGML_Q4_K
    for it in range(3):
        x = O.normal_f32(k, seed + 1 + it)
        y_ref = run_matvec(fmt, w, rows, k, x)
        xh.copy_(torch.from_numpy(x))
        A.call("arcllm_cuda_matvec_hostio", ty, G.ptr(w), rows, k, C.c_void_p(xh.data_ptr()), G.ptr(xd),
               G.ptr(yd), C.c_void_p(yh.data_ptr()), G.stream())
        assert np.array_equal(yh.numpy().view(np.uint32), y_ref.view(np.uint32)), it
    G.check_device_error()
