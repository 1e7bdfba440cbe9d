"""The allocation-free attention entry point against the regular one.

arcllm_cuda_attention_decode_noalloc exists for callers that cannot allocate
device memory at step time (fixed device-memory plans, latency-critical loops,
plugins without their own budget): it keeps the slice partials in a fixed
array inside the library instead of taking a scratch buffer.  This test calls
it through the C ABI twice in a row, with different positions, layers and
inputs, and checks each result against arcllm_cuda_attention_decode on the
same inputs with the tolerance of the other attention tests (rel-L2 1e-4),
plus the size limit.  It lives in its own file, collected last, and needs no
state from other tests.
"""
import ctypes as C

import numpy as np
import pytest

import arcllm_b200 as A
import oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
from tests import gpu_util as G  # noqa: E402

QH, KVH, D, MC, LAYERS, SPLITS = 28, 4, 128, 4096, 2, 16


def _inputs(seed, pos):
    KV = KVH * D
    kc = O.normal_f32(LAYERS * MC * KV, seed, 0.0, 1.0).astype(np.float16)
    vc = O.normal_f32(LAYERS * MC * KV, seed + 1, 0.0, 1.0).astype(np.float16)
    q = O.normal_f32(QH * D, seed + 2, 0.0, 1.0)
    return (G.to_dev(q), G.to_dev(kc.view(np.uint16)), G.to_dev(vc.view(np.uint16)),
            G.to_dev(np.array([pos], np.uint32)))


def test_noalloc_attention_matches_regular_entry_point_twice():
    for seed, pos, layer in ((300, 1000, 1), (400, 57, 0)):
        q, kc, vc, posd = _inputs(seed, pos)
        scratch = G.empty_f32(KVH * SPLITS * (QH // KVH) * (D + 2))
        ref = G.empty_f32(QH * D)
        A.call("arcllm_cuda_attention_decode", G.ptr(q), G.ptr(kc), G.ptr(vc), G.ptr(posd), QH, KVH, D, MC, layer,
               SPLITS, G.ptr(scratch), G.ptr(ref), G.stream())
        out = G.empty_f32(QH * D)
        A.call("arcllm_cuda_attention_decode_noalloc", G.ptr(q), G.ptr(kc), G.ptr(vc), G.ptr(posd), QH, KVH, D, MC,
               layer, SPLITS, G.ptr(out), G.stream())
        y, r = G.host(out).astype(np.float64), G.host(ref).astype(np.float64)
        assert np.all(np.isfinite(y))
        assert np.linalg.norm(y - r) / np.linalg.norm(r) <= 1e-4
        assert np.abs(y - r).max() <= 1e-4 * 4.0
    G.check_device_error()


def test_noalloc_attention_rejects_oversized_requests():
    q, kc, vc, posd = _inputs(500, 10)
    out = G.empty_f32(QH * D)
    L = A.lib()
    st = L.arcllm_cuda_attention_decode_noalloc(G.ptr(q), G.ptr(kc), G.ptr(vc), G.ptr(posd), QH, KVH, D, MC, 0,
                                                 64, G.ptr(out), G.stream())
    assert L.arcllm_cuda_status_string(st) == b"ARC_E_UNSUPPORTED_SHAPE"
    assert b"65536" in L.arcllm_cuda_last_error_message()
