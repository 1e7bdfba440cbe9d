"""GPU parity of the decode-step ops and of end-to-end greedy decode.

Bars: RoPE rotation and the fp16 KV-cache store bit-exact against the oracle
(the cos/sin table uses the reference's float expression); attention within
rel-L2 1e-4 of the reference's attention_cache_cpu over the same fp16-rounded
cache; greedy argmax identical to the reference's first-index rule; end-to-end
logits within rel-L2 1e-2 of the CPU oracle decode at every step, with the
greedy token-match rate reported (and required to be 1.0 on these seeds).
"""
import ctypes as C
import os

import numpy as np
import pytest

import arcllm_b200 as A
import oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
from tests import gpu_util as G  # noqa: E402
from tests.oracle_decode import OracleModel  # noqa: E402


def rope_table_dev(max_ctx, dim=128, theta=1.0e6):
    t = G.empty_f32(max_ctx * dim)
    A.call("arcllm_cuda_rope_table", G.ptr(t), max_ctx, dim, C.c_float(theta))
    return t


@pytest.mark.parametrize("pos", [0, 1, 255, 4095])
def test_rope_kv_store_bit_exact(pos):
    QH, KVH, D, MC, layers, layer = 28, 4, 128, 4096, 2, 1
    q = O.normal_f32(QH * D, 10 + pos, 0.0, 3.0)
    k = O.normal_f32(KVH * D, 11 + pos, 0.0, 3.0)
    v = O.normal_f32(KVH * D, 12 + pos, 0.0, 3.0)
    qd, kd, vd = G.to_dev(q), G.to_dev(k), G.to_dev(v)
    kc = torch.zeros(layers * MC * KVH * D, dtype=torch.int16, device=G.dev())
    vc = torch.zeros_like(kc)
    tab = rope_table_dev(MC)
    posd = G.to_dev(np.array([pos], np.uint32))
    A.call("arcllm_cuda_rope_kv_store", G.ptr(qd), G.ptr(kd), G.ptr(vd), G.ptr(tab), G.ptr(posd), G.ptr(kc), G.ptr(vc),
           QH, KVH, D, MC, layer, G.stream())
    qr = O.rope(q, QH, D, pos, 1.0e6)
    kr = O.rope(k, KVH, D, pos, 1.0e6)
    assert np.array_equal(G.host(qd).view(np.uint32), qr.view(np.uint32))
    assert np.array_equal(G.host(kd).view(np.uint32), kr.view(np.uint32))
    base = (layer * MC + pos) * KVH * D
    kch = G.host(kc).view(np.uint16)[base:base + KVH * D]
    vch = G.host(vc).view(np.uint16)[base:base + KVH * D]
    assert np.array_equal(kch, kr.astype(np.float16).view(np.uint16))
    assert np.array_equal(vch, v.astype(np.float16).view(np.uint16))
    G.check_device_error()


@pytest.mark.parametrize("pos,splits", [(0, 16), (1, 16), (37, 3), (255, 16), (1000, 64), (4095, 16), (4095, 1)])
def test_attention_decode(pos, splits):
    QH, KVH, D, MC, layers, layer = 28, 4, 128, 4096, 2, 1
    KV = KVH * D
    kc = O.normal_f32(layers * MC * KV, 20 + pos, 0.0, 1.0).astype(np.float16)
    vc = O.normal_f32(layers * MC * KV, 21 + pos, 0.0, 1.0).astype(np.float16)
    q = O.normal_f32(QH * D, 22 + pos, 0.0, 1.0)
    kcd, vcd, qd = G.to_dev(kc.view(np.uint16)), G.to_dev(vc.view(np.uint16)), G.to_dev(q)
    posd = G.to_dev(np.array([pos], np.uint32))
    scratch = G.empty_f32(KVH * splits * (QH // KVH) * (D + 2))
    out = G.empty_f32(QH * D)
    A.call("arcllm_cuda_attention_decode", G.ptr(qd), G.ptr(kcd), G.ptr(vcd), G.ptr(posd), QH, KVH, D, MC, layer,
           splits, G.ptr(scratch), G.ptr(out), G.stream())
    ref = O.attention_cache(q, kc.astype(np.float32), vc.astype(np.float32), layer, pos, MC, QH, KVH, D)
    y = G.host(out).astype(np.float64)
    rel = np.linalg.norm(y - ref) / np.linalg.norm(ref)
    assert rel <= 1e-4, rel
    assert np.abs(y - ref).max() <= 1e-4 * 4.0


@pytest.mark.parametrize("pos,splits", [(5, 16), (300, 16), (4095, 16), (37, 3), (1000, 8)])
def test_attention_cluster_merge_bit_identical(pos, splits, monkeypatch):
    """Slices merged through distributed shared memory inside their cluster
    equal the separate merge kernel's output bit for bit."""
    QH, KVH, D, MC, layers, layer = 28, 4, 128, 4096, 2, 1
    KV = KVH * D
    kc = O.normal_f32(layers * MC * KV, 40 + pos, 0.0, 1.0).astype(np.float16)
    vc = O.normal_f32(layers * MC * KV, 41 + pos, 0.0, 1.0).astype(np.float16)
    q = O.normal_f32(QH * D, 42 + pos, 0.0, 1.0)
    kcd, vcd, qd = G.to_dev(kc.view(np.uint16)), G.to_dev(vc.view(np.uint16)), G.to_dev(q)
    posd = G.to_dev(np.array([pos], np.uint32))
    scratch = G.empty_f32(KVH * splits * (QH // KVH) * (D + 2))
    outs = {}
    for flag in ("1", "0"):
        monkeypatch.setenv("ARCLLM_ATTN_CLUSTER", flag)
        out = G.empty_f32(QH * D)
        A.call("arcllm_cuda_attention_decode", G.ptr(qd), G.ptr(kcd), G.ptr(vcd), G.ptr(posd), QH, KVH, D, MC,
               layer, splits, G.ptr(scratch), G.ptr(out), G.stream())
        outs[flag] = G.host(out)
    assert np.array_equal(outs["1"].view(np.uint32), outs["0"].view(np.uint32))
    G.check_device_error()


@pytest.mark.parametrize("etype", [A.GGML_F16, A.GGML_Q4_K])
def test_embed(etype):
    V, H, tok = 1000, 512, 777
    if etype == A.GGML_F16:
        tab = O.normal_f16(V * H, 5, 0.0, 0.02)
        ref = tab[tok * H:(tok + 1) * H].view(np.float16).astype(np.float32)
    else:
        tab = O.fill_q4k(V, H, 5)
        rb = (H // 256) * 144
        ref = O.dequant("q4k", tab[tok * rb:(tok + 1) * rb], 1, H).ravel()
    td = G.to_dev(tab)
    tokd = G.to_dev(np.array([tok], np.uint32))
    out = G.empty_f32(H)
    A.call("arcllm_cuda_embed", etype, G.ptr(td), G.ptr(tokd), H, V, G.ptr(out), G.stream())
    assert np.array_equal(G.host(out).view(np.uint32), ref.view(np.uint32))


def test_argmax_reference_rule(golden):
    scratch = torch.zeros(4, dtype=torch.int32, device=G.dev())
    L = A.lib()

    def run(x):
        xd = G.to_dev(np.ascontiguousarray(x, np.float32))
        idx, fin = C.c_uint32(0), C.c_int(0)
        A.call("arcllm_cuda_argmax", G.ptr(xd), x.size, G.ptr(scratch), C.byref(idx), C.byref(fin), G.stream())
        return idx.value, fin.value

    cases = [np.array([1, 3, 3, 2], np.float32), np.array([-5, -1, -1, -7], np.float32),
             O.normal_f32(152064, 0x41), np.full(300000, 2.5, np.float32), np.array([-0.0, 0.0], np.float32)]
    for x in cases:
        i_ref, fin_ref = O.argmax(x)
        assert run(x) == (i_ref, int(fin_ref))
    # non-finite logits are flagged (the runtime then refuses: runtime.cpp:446,501)
    assert run(np.array([0, np.nan, 4, 4], np.float32))[1] == 0
    assert run(np.array([np.inf, 1, 2], np.float32))[1] == 0
    del L


SMALL = dict(n_layers=2, hidden=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn=1024, vocab=4096, max_ctx=64,
             rms_eps=1e-6, rope_theta=1.0e6)


def run_parity(cfg, prompt, n_new, types=None, threads=8):
    from arcllm_b200.synthetic import SyntheticModel
    m = SyntheticModel(cfg, types=types, seed=0x5EED + cfg["n_layers"])
    ref = OracleModel(m.cfg, m.specs, threads=threads)
    m.begin(prompt, n_new)
    toks, rels, match = list(prompt), [], 0
    pos = 0
    # teacher-forced: both sides consume the same token sequence
    for step in range(len(prompt) + n_new - 1):
        m.step(with_head=True, use_graph=(step % 2 == 1))
        yg = m.logits()
        yr = ref.step(toks[pos], pos)
        rels.append(float(np.linalg.norm(yg.astype(np.float64) - yr) / np.linalg.norm(yr)))
        if pos + 1 >= len(prompt):
            tg, _ = O.argmax(yg)
            tr, _ = O.argmax(yr)
            match += int(tg == tr)
            toks.append(tg)
        pos += 1
    G.check_device_error()
    m.close()
    return rels, match / n_new, toks[len(prompt):]


def test_decode_small_model_parity():
    prompt = [int(t) for t in O.tokens(8, 0x77, SMALL["vocab"])]
    rels, rate, _ = run_parity(SMALL, prompt, 8)
    print("small model: max rel-L2 %.2e, token match %.2f" % (max(rels), rate))
    assert max(rels) <= 1e-2
    assert rate == 1.0


def test_decode_small_q4_everywhere():
    types = dict(wv=A.GGML_Q4_K, w_down=A.GGML_Q4_K, output=A.GGML_Q4_K, tok_embd=A.GGML_Q4_K)
    prompt = [int(t) for t in O.tokens(5, 0x78, SMALL["vocab"])]
    rels, rate, _ = run_parity(SMALL, prompt, 4, types=types)
    assert max(rels) <= 1e-2 and rate == 1.0


def test_generate_matches_stepwise_and_reports_stats():
    from arcllm_b200.synthetic import SyntheticModel
    m = SyntheticModel(SMALL, seed=0x5EED + 2)
    m.set_prefill_mode(0)  # token by token: the same fp32 chain as the eager steps below
    prompt = [int(t) for t in O.tokens(8, 0x77, SMALL["vocab"])]
    toks, st = m.generate(prompt, 8)
    toks2, st2 = m.generate(prompt, 8)  # request-scoped: a second request repeats exactly
    assert toks == toks2
    m.begin(prompt, 8)
    ref = []
    for i in range(len(prompt) + 7):
        m.step(with_head=True, use_graph=False)
        if i + 1 >= len(prompt):
            ref.append(O.argmax(m.logits())[0])
    assert toks == ref
    assert st.finite == 1 and st.decode_steps == 7 and st.prefill_graph_launches == 8
    # RoPE + KV store fused into Q/K/V, Q/K/V in one launch (three with ARCLLM_QKV_ONE_LAUNCH=0),
    # attention slices merged inside their cluster
    per_layer = 7 if os.environ.get("ARCLLM_QKV_ONE_LAUNCH") == "0" else 5
    assert st.decode_launches_per_step == 1 + per_layer * SMALL["n_layers"] + 3
    assert st.decode_graph_launches_per_step == 1
    m.close()


def test_decode_qwen7b_shape_parity():
    """The full Qwen2.5-7B layer shapes (hidden 3584, 28/4 heads, ffn 18944,
    vocab 152064), two layers so the CPU oracle stays fast."""
    cfg = dict(n_layers=2, hidden=3584, n_heads=28, n_kv_heads=4, head_dim=128, ffn=18944, vocab=152064,
               max_ctx=4096, rms_eps=1e-6, rope_theta=1.0e6)
    prompt = [int(t) for t in O.tokens(3, 0x79, cfg["vocab"])]
    rels, rate, _ = run_parity(cfg, prompt, 3, threads=max(8, os.cpu_count() or 8))
    print("7B-shape: max rel-L2 %.2e, token match %.2f" % (max(rels), rate))
    assert max(rels) <= 1e-2 and rate == 1.0


def test_fused_rope_kv_epilogue_bit_identical(monkeypatch):
    """RoPE and the fp16 KV store in the Q/K/V matvec epilogues give the same
    cache and logits, bit for bit, as the separate rope_kv_store kernel."""
    from arcllm_b200.synthetic import SyntheticModel
    prompt = [int(t) for t in O.tokens(9, 0x7E, SMALL["vocab"])]
    out = {}
    for fused in ("1", "0"):
        monkeypatch.setenv("ARCLLM_FUSE_ROPE", fused)
        m = SyntheticModel(SMALL, seed=0x5EED + 13)
        m.set_prefill_mode(0)
        toks, st = m.generate(prompt, 5)
        n = len(prompt) + 4
        out[fused] = (toks, st.decode_launches_per_step, m.logits(), [m.kv_cache(l, n) for l in range(2)])
        m.close()
    a, b = out["1"], out["0"]
    assert a[0] == b[0]
    fused_per_layer = 7 if os.environ.get("ARCLLM_QKV_ONE_LAUNCH") == "0" else 5  # Q/K/V in one launch
    assert a[1] == 1 + fused_per_layer * SMALL["n_layers"] + 3 and b[1] == 1 + 8 * SMALL["n_layers"] + 3
    assert np.array_equal(a[2].view(np.uint32), b[2].view(np.uint32))
    for l in range(2):
        for j in range(2):
            assert np.array_equal(a[3][l][j].view(np.uint16), b[3][l][j].view(np.uint16))
    G.check_device_error()
