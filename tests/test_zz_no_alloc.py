"""The allocation-free attention entry point against the regular one.

arcllm_cuda_attention_decode_noalloc exists for callers that cannot allocate
device memory at step time (fixed device-memory plans, latency-critical loops,
plugins without their own budget): it keeps the slice partials in a fixed
array inside the library instead of taking a scratch buffer.

The partials pass through that array only when the slices are merged by the
separate merge kernel: with the clustered form (2..16 slices per KV head on a
device that schedules such clusters) the slices merge through distributed
shared memory and no scratch is touched.  So the cases here take the
two-kernel form on purpose -- 17 slices (past the 16-CTA cluster limit), and
16 slices with ARCLLM_ATTN_CLUSTER=0 -- and one clustered case checks that the
entry point also works when the array is not in play.  Each case calls the
entry point through the C ABI twice in a row (different positions, layers and
inputs, so the second call overwrites what the first left in the array) and
requires bit identity with arcllm_cuda_attention_decode given caller scratch
on the same path, and rel-L2 <= 1e-4 against the reference's
attention_cache_cpu restated in the oracle.  The file is collected last and
needs no state from other tests.
"""
import ctypes as C

import numpy as np
import pytest

import arcllm_b200 as A
import oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
from tests import gpu_util as G  # noqa: E402

QH, KVH, D, MC, LAYERS = 28, 4, 128, 4096, 2


def _inputs(seed, pos):
    KV = KVH * D
    kc = O.normal_f32(LAYERS * MC * KV, seed, 0.0, 1.0).astype(np.float16)
    vc = O.normal_f32(LAYERS * MC * KV, seed + 1, 0.0, 1.0).astype(np.float16)
    q = O.normal_f32(QH * D, seed + 2, 0.0, 1.0)
    dev = (G.to_dev(q), G.to_dev(kc.view(np.uint16)), G.to_dev(vc.view(np.uint16)),
           G.to_dev(np.array([pos], np.uint32)))
    return dev, (q, kc, vc)


@pytest.mark.parametrize("splits,cluster", [(17, "1"), (16, "0"), (16, "1")],
                         ids=["17-splits-merge-kernel", "16-splits-cluster-off", "16-splits-clustered"])
def test_noalloc_attention_matches_regular_entry_point_twice(splits, cluster, monkeypatch):
    monkeypatch.setenv("ARCLLM_ATTN_CLUSTER", cluster)
    assert KVH * splits * (QH // KVH) * (D + 2) <= 65536
    for seed, pos, layer in ((300, 1000, 1), (400, 57, 0)):
        (q, kc, vc, posd), (qh, kch, vch) = _inputs(seed + splits, pos)
        scratch = G.empty_f32(KVH * splits * (QH // KVH) * (D + 2))
        ref = G.empty_f32(QH * D)
        A.call("arcllm_cuda_attention_decode", G.ptr(q), G.ptr(kc), G.ptr(vc), G.ptr(posd), QH, KVH, D, MC, layer,
               splits, G.ptr(scratch), G.ptr(ref), G.stream())
        out = G.empty_f32(QH * D)
        A.call("arcllm_cuda_attention_decode_noalloc", G.ptr(q), G.ptr(kc), G.ptr(vc), G.ptr(posd), QH, KVH, D, MC,
               layer, splits, G.ptr(out), G.stream())
        y, r = G.host(out), G.host(ref)
        assert np.all(np.isfinite(y))
        assert np.array_equal(y.view(np.uint32), r.view(np.uint32))
        want = O.attention_cache(qh, kch.astype(np.float32), vch.astype(np.float32), layer, pos, MC, QH, KVH, D)
        y64 = y.astype(np.float64)
        assert np.linalg.norm(y64 - want) / np.linalg.norm(want) <= 1e-4
    G.check_device_error()


def test_noalloc_attention_rejects_oversized_requests():
    (q, kc, vc, posd), _ = _inputs(500, 10)
    out = G.empty_f32(QH * D)
    L = A.lib()
    st = L.arcllm_cuda_attention_decode_noalloc(G.ptr(q), G.ptr(kc), G.ptr(vc), G.ptr(posd), QH, KVH, D, MC, 0,
                                                 64, G.ptr(out), G.stream())
    assert L.arcllm_cuda_status_string(st) == b"ARC_E_UNSUPPORTED_SHAPE"
    assert b"65536" in L.arcllm_cuda_last_error_message()
