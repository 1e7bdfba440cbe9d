"""Prefill GEMM on tcgen05 (arcllm_cuda_gemm_q4k_bf16 / arcllm_cuda_gemm_bf16 /
arcllm_cuda_gemm_f16): y = (residual +) x * W^T with x bf16 (fp16) [m x k],
W Q4_K or Q6_K [n x k], fp32 accumulation.  Checked tightly against the same
product with W dequantised the way the kernel does it (bf16 or fp16 scale and
offset per sub-block, one rounding of q*f - o), and at the stated 1e-2 rel-L2
(6e-4 for the fp16 form) against the CPU oracle's bit-exact fp32
dequantisation; plus the batched RMSNorm that produces x."""
import ctypes as C

import numpy as np
import pytest
import torch

import arcllm_b200 as A
import oracle as O
import gpu_util as G

pytestmark = pytest.mark.gpu


def bf16_round(a, dt=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dt).to(torch.float32).numpy()


def q4k_bf16_weights(w_host, n, k, dt=torch.bfloat16):
    """The kernel's bf16 (or fp16, dt) weights: f = rnd(d*sc), o = rnd(dmin*mn)
    per sub-block, w = rnd(q*f - o) with one rounding."""
    nb = k // 256
    blk = w_host.reshape(n * nb, 144)
    d = blk[:, 0:2].copy().view(np.float16).astype(np.float32)[:, 0]
    dmin = blk[:, 2:4].copy().view(np.float16).astype(np.float32)[:, 0]
    s = blk[:, 4:16].astype(np.int32)
    sc = np.empty((n * nb, 8), np.int32)
    mn = np.empty((n * nb, 8), np.int32)
    for j in range(8):
        if j < 4:
            sc[:, j] = s[:, j] & 63
            mn[:, j] = s[:, j + 4] & 63
        else:
            sc[:, j] = (s[:, j + 4] & 15) | ((s[:, j - 4] >> 6) << 4)
            mn[:, j] = (s[:, j + 4] >> 4) | ((s[:, j] >> 6) << 4)
    f = bf16_round((d[:, None] * sc.astype(np.float32)).astype(np.float32), dt).astype(np.float64)
    o = bf16_round((dmin[:, None] * mn.astype(np.float32)).astype(np.float32), dt).astype(np.float64)
    kk = np.arange(256)
    byte = blk[:, 16 + (kk >> 6) * 32 + (kk & 31)].astype(np.int32)
    q = np.where((kk & 63) < 32, byte & 15, byte >> 4).astype(np.float64)
    w = q * f[:, kk >> 5] - o[:, kk >> 5]
    return bf16_round(w.astype(np.float32), dt).reshape(n, k)


def q6k_bf16_weights(w_host, n, k, dt=torch.bfloat16):
    """The kernel's bf16 (or fp16, dt) Q6_K weights: f = rnd(d*sc) per
    16-element group, w = rnd((c - 32) * f) with one rounding."""
    nb = k // 256
    blk = w_host.reshape(n * nb, 210)
    d = blk[:, 208:210].copy().view(np.float16).astype(np.float32)[:, 0]
    sc = blk[:, 192:208].astype(np.int8).astype(np.float32)
    f = bf16_round((d[:, None] * sc).astype(np.float32), dt).astype(np.float64)
    kk = np.arange(256)
    h, q, l = kk >> 7, (kk & 127) >> 5, kk & 31
    low = (blk[:, 64 * h + 32 * (q & 1) + l].astype(np.int32) >> (4 * (q >> 1))) & 15
    high = (blk[:, 128 + 32 * h + l].astype(np.int32) >> (2 * q)) & 3
    c = (low | (high << 4)).astype(np.float64) - 32.0
    w = c * f[:, 8 * h + 2 * q + (l >> 4)]
    return bf16_round(w.astype(np.float32), dt).reshape(n, k)


def run_gemm_t(fmt, m, n, k, seed, residual=False):
    w_host = O.fill_weights(fmt, n, k, seed)
    w = G.to_dev(w_host)
    x32 = O.normal_f32(m * k, seed + 1).reshape(m, k)
    xb = torch.from_numpy(x32).to(torch.bfloat16).to(G.dev())
    r = torch.from_numpy(O.normal_f32(m * n, seed + 2).reshape(m, n)).to(G.dev()) if residual else None
    y = torch.full((m, n), float("nan"), dtype=torch.float32, device=G.dev())
    A.call("arcllm_cuda_gemm_bf16", 12 if fmt == "q4k" else 14, G.ptr(w), n, k, C.c_void_p(xb.data_ptr()), m,
           C.c_void_p(r.data_ptr()) if residual else None, C.c_void_p(y.data_ptr()), G.stream())
    torch.cuda.synchronize()
    G.check_device_error()
    wd = O.dequant(fmt, w_host, n, k).reshape(n, k)
    wb = q4k_bf16_weights(w_host, n, k) if fmt == "q4k" else q6k_bf16_weights(w_host, n, k)
    xf = xb.float().cpu().numpy().astype(np.float64)
    rr = r.cpu().numpy().astype(np.float64) if residual else 0.0
    return y.cpu().numpy().astype(np.float64), xf, wd, wb, rr


@pytest.mark.parametrize("fmt,m,n,k,res", [("q6k", 256, 128, 256, False), ("q6k", 255, 512, 3584, True),
                                           ("q6k", 100, 384, 1024, False), ("q6k", 256, 3584, 18944, True),
                                           ("q6k", 1, 128, 512, True), ("q4k", 255, 3584, 3584, True),
                                           ("q4k", 64, 3584, 18944, True)])
def test_gemm_bf16_formats_and_residual(fmt, m, n, k, res):
    y, xf, wd, wb, rr = run_gemm_t(fmt, m, n, k, 1300 + m + n + k, res)
    assert np.isfinite(y).all()
    y_b = rr + xf @ wb.astype(np.float64).T
    y_f = rr + xf @ wd.astype(np.float64).T
    rel_b = np.linalg.norm(y - y_b) / np.linalg.norm(y_b)
    rel_f = np.linalg.norm(y - y_f) / np.linalg.norm(y_f)
    print("gemm %s %dx%dx%d res=%d: rel-L2 %.2e (kernel's bf16 W), %.2e (fp32 W)" % (fmt, m, n, k, res, rel_b, rel_f))
    assert rel_b <= 1e-5
    assert rel_f <= 1e-2


def run_gemm(m, n, k, seed):
    w_host = O.fill_weights("q4k", n, k, seed)
    w = G.to_dev(w_host)
    x32 = O.normal_f32(m * k, seed + 1).reshape(m, k)
    xb = torch.from_numpy(x32).to(torch.bfloat16).to(G.dev())
    y = torch.full((m, n), float("nan"), dtype=torch.float32, device=G.dev())
    A.call("arcllm_cuda_gemm_q4k_bf16", G.ptr(w), n, k, C.c_void_p(xb.data_ptr()), m, C.c_void_p(y.data_ptr()),
           G.stream())
    torch.cuda.synchronize()
    G.check_device_error()
    wd = O.dequant("q4k", w_host, n, k).reshape(n, k)
    xf = xb.float().cpu().numpy().astype(np.float64)
    return y.cpu().numpy().astype(np.float64), xf, wd, q4k_bf16_weights(w_host, n, k)


@pytest.mark.parametrize("m,n,k", [(256, 128, 256), (256, 384, 3584), (100, 256, 1024), (1, 128, 512),
                                   (256, 18944, 3584),
                                   # split-K: the FFN-down shape (28 column tiles x 5 splits), many small splits
                                   (256, 3584, 18944), (64, 256, 2048), (1, 128, 4096)])
def test_gemm_q4k_bf16(m, n, k):
    y, xf, wd, wb = run_gemm(m, n, k, 900 + m + n + k)
    assert np.isfinite(y).all()
    y_b = xf @ wb.astype(np.float64).T                  # what the tensor cores compute
    y_f = xf @ wd.astype(np.float64).T                  # fp32 dequantised weights (the reference's)
    rel_b = np.linalg.norm(y - y_b) / np.linalg.norm(y_b)
    rel_f = np.linalg.norm(y - y_f) / np.linalg.norm(y_f)
    print("gemm %dx%dx%d: rel-L2 %.2e (kernel's bf16 W), %.2e (fp32 W)" % (m, n, k, rel_b, rel_f))
    assert rel_b <= 1e-5
    assert rel_f <= 1e-2


def test_gemm_rejects_bad_shapes():
    L = A.lib()
    w = G.empty_u8(144 * 2 * 128)
    x = torch.zeros(256 * 512, dtype=torch.bfloat16, device=G.dev())
    y = G.empty_f32(256 * 128)
    args = lambda m, n, k: (G.ptr(w), n, k, C.c_void_p(x.data_ptr()), m, G.ptr(y), G.stream())  # noqa: E731
    for m, n, k in ((257, 128, 512), (0, 128, 512), (256, 100, 512), (256, 128, 300)):
        st = L.arcllm_cuda_gemm_q4k_bf16(*args(m, n, k))
        assert L.arcllm_cuda_status_string(st) == b"ARC_E_UNSUPPORTED_SHAPE"



@pytest.mark.parametrize("fmt,m,n,k,res", [("q4k", 255, 3584, 3584, False), ("q4k", 255, 512, 3584, False),
                                           ("q6k", 255, 512, 3584, True), ("q4k", 100, 384, 1024, True),
                                           ("q6k", 256, 3584, 18944, False), ("q4k", 1, 128, 512, False)])
def test_gemm_f16_operands(fmt, m, n, k, res):
    """arcllm_cuda_gemm_f16: fp16 x times the weights dequantised to fp16 (the
    kernel's rounding: f, o and q*f - o each to fp16).  Within 1e-5 of that
    product, and about 8x closer to the fp32-dequantised product than the
    bf16 GEMM (the Q/K/V projections of the prefill use it)."""
    seed = 2300 + m + n + k
    w_host = O.fill_weights(fmt, n, k, seed)
    w = G.to_dev(w_host)
    x32 = O.normal_f32(m * k, seed + 1).reshape(m, k)
    xh = torch.from_numpy(x32).to(torch.float16).to(G.dev())
    r = torch.from_numpy(O.normal_f32(m * n, seed + 2).reshape(m, n)).to(G.dev()) if res else None
    y = torch.full((m, n), float("nan"), dtype=torch.float32, device=G.dev())
    A.call("arcllm_cuda_gemm_f16", 12 if fmt == "q4k" else 14, G.ptr(w), n, k, C.c_void_p(xh.data_ptr()), m,
           C.c_void_p(r.data_ptr()) if res else None, C.c_void_p(y.data_ptr()), G.stream())
    torch.cuda.synchronize()
    G.check_device_error()
    yv = y.cpu().numpy().astype(np.float64)
    wf = (q4k_bf16_weights if fmt == "q4k" else q6k_bf16_weights)(w_host, n, k, torch.float16).astype(np.float64)
    wd = O.dequant(fmt, w_host, n, k).reshape(n, k).astype(np.float64)
    rr = r.cpu().numpy().astype(np.float64) if res else 0.0
    xf = xh.float().cpu().numpy().astype(np.float64)
    y_k = rr + xf @ wf.T
    y_f = x32.astype(np.float64) @ wd.T
    rel_k = np.linalg.norm(yv - y_k) / np.linalg.norm(y_k)
    rel_f = np.linalg.norm(yv - rr - y_f) / np.linalg.norm(y_f)
    print("f16 gemm %s %dx%dx%d res=%d: rel-L2 %.2e (kernel's fp16 W), %.2e (fp32 x and W)"
          % (fmt, m, n, k, res, rel_k, rel_f))
    assert np.isfinite(yv).all()
    assert rel_k <= 1e-5
    assert rel_f <= 6e-4


@pytest.mark.parametrize("fp16", [0, 1])
def test_rmsnorm_rows(fp16):
    """arcllm_cuda_rmsnorm_rows: v = x * rsqrt(mean(x^2) + eps) * gamma per row
    (sum of squares in double), rounded to bf16 or fp16."""
    rows, h, eps = 37, 3584, 1e-6
    x = O.normal_f32(rows * h, 77, 0.0, 3.0).reshape(rows, h)
    g = O.normal_f32(h, 78, 1.0, 0.1)
    xd, gd = G.to_dev(x), G.to_dev(g)
    out = torch.empty(rows * h, dtype=torch.int16, device=G.dev())
    lo = torch.zeros(rows * h, dtype=torch.int16, device=G.dev()) if fp16 else None
    A.call("arcllm_cuda_rmsnorm_rows", G.ptr(xd), G.ptr(gd), C.c_float(eps), rows, h, fp16, G.ptr(out), G.ptr(lo),
           G.stream())
    raw = G.host(out).view(np.uint16)
    got = raw.view(np.float16).astype(np.float32) if fp16 else (raw.astype(np.uint32) << 16).view(np.float32)
    ss = (x.astype(np.float64) ** 2).sum(axis=1)
    inv = (np.float32(1.0) / np.sqrt((ss / h).astype(np.float32) + np.float32(eps))).astype(np.float32)
    v = ((x * inv[:, None]).astype(np.float32) * g[None, :]).astype(np.float32)
    want = bf16_round(v, torch.float16 if fp16 else torch.bfloat16)
    assert np.mean(got.reshape(rows, h) == want) > 0.999
    assert np.abs(got.reshape(rows, h) - v).max() <= 2.0 ** (-10 if fp16 else -7) * np.abs(v).max()
    if fp16:  # hi + lo carries ~22 bits of v
        lv = G.host(lo).view(np.uint16).view(np.float16).astype(np.float64).reshape(rows, h)
        err = np.abs(got.reshape(rows, h).astype(np.float64) + lv - v)
        assert err.max() <= 2.0 ** -20 * np.abs(v).max()
    G.check_device_error()


@pytest.mark.parametrize("fmt,m,n,k,res", [("q4k", 255, 3584, 3584, False), ("q4k", 255, 512, 3584, True),
                                           ("q6k", 255, 512, 3584, False), ("q6k", 100, 384, 1024, True),
                                           ("q4k", 256, 128, 18944, False), ("q4k", 1, 128, 512, False)])
def test_gemm_f16x3_near_fp32(fmt, m, n, k, res):
    """arcllm_cuda_gemm_f16x3: fp16 hi + lo halves of the activation and of the
    exactly dequantised weights, three products into fp32.  Within 5e-6 of the
    fp32-activation, fp32-weight product (measured 1e-6 to 2.7e-6; the bf16
    form is ~2.4e-3 from it, the single-fp16 form ~3.6e-4)."""
    seed = 2500 + m + n + k
    w_host = O.fill_weights(fmt, n, k, seed)
    w = G.to_dev(w_host)
    x32 = O.normal_f32(m * k, seed + 1).reshape(m, k)
    xh = torch.from_numpy(x32).to(torch.float16)
    xl = torch.from_numpy((x32 - xh.float().numpy()).astype(np.float32)).to(torch.float16)
    xh, xl = xh.to(G.dev()), xl.to(G.dev())
    r = torch.from_numpy(O.normal_f32(m * n, seed + 2).reshape(m, n)).to(G.dev()) if res else None
    y = torch.full((m, n), float("nan"), dtype=torch.float32, device=G.dev())
    A.call("arcllm_cuda_gemm_f16x3", 12 if fmt == "q4k" else 14, G.ptr(w), n, k, C.c_void_p(xh.data_ptr()),
           C.c_void_p(xl.data_ptr()), m, C.c_void_p(r.data_ptr()) if res else None, C.c_void_p(y.data_ptr()),
           G.stream())
    torch.cuda.synchronize()
    G.check_device_error()
    yv = y.cpu().numpy().astype(np.float64)
    wd = O.dequant(fmt, w_host, n, k).reshape(n, k).astype(np.float64)
    rr = r.cpu().numpy().astype(np.float64) if res else 0.0
    y_f = x32.astype(np.float64) @ wd.T
    rel = np.linalg.norm(yv - rr - y_f) / np.linalg.norm(y_f)
    print("f16x3 gemm %s %dx%dx%d res=%d: rel-L2 %.2e vs fp32 x and W" % (fmt, m, n, k, res, rel))
    assert np.isfinite(yv).all()
    assert rel <= 5e-6


def test_prefill_chain_with_launch_overlap_equals_plain():
    """With launch overlap on (programmatic dependent launch), a kernel may start while the one before
    it runs; the matvec releases its dependents as it starts.  A chain matvec -> batched RMSNorm to
    bf16 -> split-K GEMM (+ its reduce) must still read each input only once it is complete: the
    results equal the plainly launched chain bit for bit, over repeated runs."""
    m, h, n = 64, 1024, 512
    sp = G.stream()
    wm = G.empty_u8(m * h * (h // 256) * 144 + 16)  # matvec weights: m*h rows of k = h
    A.call("arcllm_cuda_fill_q4k", G.ptr(wm), 0, m * h * (h // 256), 0x5A1, sp)
    wg = G.empty_u8(n * (h // 256) * 144 + 16)
    A.call("arcllm_cuda_fill_q4k", G.ptr(wg), 0, n * (h // 256), 0x5A2, sp)
    gamma = G.empty_f32(h)
    A.call("arcllm_cuda_fill_normal_f32", G.ptr(gamma), 0, h, 0x5A3, C.c_float(1.0), C.c_float(0.1), sp)
    xs = [G.empty_f32(h) for _ in range(3)]
    for i, x in enumerate(xs):
        A.call("arcllm_cuda_fill_normal_f32", G.ptr(x), 0, h, 0x5B0 + i, C.c_float(0.0), C.c_float(1.0), sp)
    rows = G.empty_f32(m * h)
    xb = torch.empty(m * h, dtype=torch.bfloat16, device=G.dev())
    y = G.empty_f32(m * n)

    def chain(x):
        A.call("arcllm_cuda_matvec", A.GGML_Q4_K, G.ptr(wm), m * h, h, G.ptr(x), None, C.c_float(0.0), None, None,
               G.ptr(rows), sp)
        A.call("arcllm_cuda_rmsnorm_rows", G.ptr(rows), G.ptr(gamma), C.c_float(1e-6), m, h, 0,
               C.c_void_p(xb.data_ptr()), None, sp)
        A.call("arcllm_cuda_gemm_bf16", A.GGML_Q4_K, G.ptr(wg), n, h, C.c_void_p(xb.data_ptr()), m, None, G.ptr(y), sp)

    plain = []
    for x in xs:
        chain(x)
        plain.append(G.host(y).copy())
    A.call("arcllm_cuda_set_launch_overlap", 1)
    try:
        for _ in range(3):
            for x, want in zip(xs, plain):
                y.fill_(float("nan"))
                chain(x)
                assert np.array_equal(G.host(y).view(np.uint32), want.view(np.uint32))
    finally:
        A.call("arcllm_cuda_set_launch_overlap", 0)
    G.check_device_error()
