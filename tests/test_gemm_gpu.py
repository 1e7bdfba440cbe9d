"""Prefill GEMM on tcgen05 (arcllm_cuda_gemm_q4k_bf16): y = x * W^T with x bf16
[m x k], W Q4_K [n x k], fp32 accumulation.  Checked against the CPU oracle's
bit-exact Q4_K dequantisation: tightly against the same product with W rounded
to bf16 (what the tensor cores multiply), and at the row's stated 1e-2 rel-L2
against the fp32 dequantised weights."""
import ctypes as C

import numpy as np
import pytest
import torch

import arcllm_b200 as A
import oracle as O
import gpu_util as G

pytestmark = pytest.mark.gpu


def bf16_round(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16).to(torch.float32).numpy()


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
    return y.cpu().numpy().astype(np.float64), xf, wd


@pytest.mark.parametrize("m,n,k", [(256, 128, 256), (256, 384, 3584), (100, 256, 1024), (1, 128, 512),
                                   (256, 18944, 3584)])
def test_gemm_q4k_bf16(m, n, k):
    y, xf, wd = run_gemm(m, n, k, 900 + m + n + k)
    assert np.isfinite(y).all()
    y_b = xf @ bf16_round(wd).astype(np.float64).T      # what the tensor cores compute
    y_f = xf @ wd.astype(np.float64).T                  # fp32 dequantised weights (the reference's)
    rel_b = np.linalg.norm(y - y_b) / np.linalg.norm(y_b)
    rel_f = np.linalg.norm(y - y_f) / np.linalg.norm(y_f)
    print("gemm %dx%dx%d: rel-L2 %.2e (bf16 W), %.2e (fp32 W)" % (m, n, k, rel_b, rel_f))
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
