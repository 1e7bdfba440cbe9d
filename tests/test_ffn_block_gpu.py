"""The decode FFN block through its C-ABI entry (arcllm_cuda_ffn_block) at the
Qwen2.5-7B shape (hidden 3584, ffn 18944), Q6_K and Q4_K down projections:

* bit for bit the explicit two-launch form (arcllm_cuda_gateup_silu_q4k, then
  the down projection with the residual through arcllm_cuda_matvec), for s
  and for y;
* back-to-back calls give the same bits (the split-K kernel's launch tags
  move on: no stale partial word is taken for a new one);
* against the CPU oracle's RMSNorm -> gate/up -> SwiGLU -> down + residual
  (src/arcllm_v1_runtime.cpp:389-415) within the matvec bars.
"""
import ctypes as C

import numpy as np
import pytest

import arcllm_b200 as A
import oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
from tests import gpu_util as G  # noqa: E402

H, F = 3584, 18944
BS = {"q4k": A.Q4K_BLOCK_BYTES, "q6k": A.Q6K_BLOCK_BYTES}
TY = {"q4k": A.GGML_Q4_K, "q6k": A.GGML_Q6_K}


def _fill(fmt, rows, k, seed):
    nb = k // 256
    t = G.empty_u8(rows * nb * BS[fmt] + 16)
    A.call("arcllm_cuda_fill_" + fmt, G.ptr(t), 0, rows * nb, seed, G.stream())
    return t


def _bits(t):
    return G.host(t).view(np.uint32)


@pytest.mark.parametrize("down", ["q6k", "q4k"])
def test_ffn_block_equals_two_launches_and_oracle(down):
    seed = 0xF00 + (6 if down == "q6k" else 4)
    wg, wu = _fill("q4k", F, H, seed), _fill("q4k", F, H, seed + 1)
    wd = _fill(down, H, F, seed + 2)
    x = O.normal_f32(H, seed + 3)
    gamma = O.normal_f32(H, seed + 4, 1.0, 0.1)
    res = O.normal_f32(H, seed + 5)
    xd, gd, rd = G.to_dev(x), G.to_dev(gamma), G.to_dev(res)
    eps = C.c_float(1e-6)

    s2, y2 = G.empty_f32(F), G.empty_f32(H)  # the two-launch form
    A.call("arcllm_cuda_gateup_silu_q4k", G.ptr(wg), G.ptr(wu), F, H, G.ptr(xd), G.ptr(gd), eps, G.ptr(s2), G.stream())
    A.call("arcllm_cuda_matvec", TY[down], G.ptr(wd), H, F, G.ptr(s2), None, C.c_float(0.0), None, G.ptr(rd),
           G.ptr(y2), G.stream())
    outs = []
    for _ in range(3):
        s1, y1 = G.empty_f32(F), G.empty_f32(H)
        s1.fill_(float("nan"))
        y1.fill_(float("nan"))
        A.call("arcllm_cuda_ffn_block", TY[down], G.ptr(wg), G.ptr(wu), G.ptr(wd), H, F, G.ptr(xd), G.ptr(gd), eps,
               G.ptr(s1), G.ptr(rd), G.ptr(y1), G.stream())
        outs.append((_bits(s1), _bits(y1)))
    G.check_device_error()
    for sb, yb in outs:
        assert np.array_equal(sb, _bits(s2)), "s differs from the two-launch form"
        assert np.array_equal(yb, _bits(y2)), "y differs from the two-launch form"

    # oracle: RMSNorm -> gate/up -> SwiGLU -> down + residual
    xn = O.rmsnorm(x, gamma, 1e-6)
    g = O.matvec("q4k", O.fill_q4k(F, H, seed), F, H, xn, threads=8)
    u = O.matvec("q4k", O.fill_q4k(F, H, seed + 1), F, H, xn, threads=8)
    s_ref = O.swiglu(g, u)
    s_out = outs[0][0].view(np.float32).astype(np.float64)
    assert np.linalg.norm(s_out - s_ref) / np.linalg.norm(s_ref) <= 1e-3
    w_host = O.fill_weights(down, H, F, seed + 2)
    y_ref = O.matvec(down, w_host, H, F, s_ref.astype(np.float32), threads=8).astype(np.float64) + res
    y_out = outs[0][1].view(np.float32).astype(np.float64)
    assert np.linalg.norm(y_out - y_ref) / np.linalg.norm(y_ref) <= 1e-3
