"""Config 3 end to end: greedy decode of the Qwen2.5-7B-shaped model with all
28 layers (q/k/o/gate/up Q4_K; v, down and the LM head Q6_K; fp16 embedding
and KV cache) -- the bench's decode model (seed 0xC3) and the first 16 tokens
of its prompt stream -- against the CPU oracle's fp32 forward pass
(tests/oracle_decode.py, the order of src/arcllm_v1_runtime.cpp:371-421),
with its cache rows rounded to fp16 as the model's cache holds them.

The prompt goes through the default batched tensor-core prefill (15 rows),
then five decode steps run as the captured step graph.  The oracle steps
through the same tokens: the prompt, then at every step the token the GPU
chose (teacher-forced, so one disagreement cannot cascade).  Bars: logits
within rel-L2 1e-2 of the oracle at every step (the end-to-end tolerance);
the greedy token-match rate is printed and must be 1.0 on this seed."""
import os

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
from tests import gpu_util as G  # noqa: E402
from tests.oracle_decode import OracleModel  # noqa: E402

N_PROMPT, N_NEW = 16, 5


def bench_prompt(n, vocab, seed=0x70C):
    from arcllm_b200.synthetic import splitmix64_at
    return [int(((splitmix64_at(seed, i) >> 32) * vocab) >> 32) for i in range(n)]


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def test_config3_28_layers_batched_prefill_then_decode_against_oracle():
    from arcllm_b200.synthetic import QWEN25_7B, SyntheticModel
    cfg = dict(QWEN25_7B)
    prompt = bench_prompt(N_PROMPT, cfg["vocab"])
    m = SyntheticModel(cfg, seed=0xC3)
    m.begin(prompt, N_NEW)
    m.prefill()
    logits, toks = [], []
    for _ in range(N_NEW):
        m.step(with_head=True, use_graph=True)
        lg = m.logits()
        logits.append(lg)
        toks.append(O.argmax(lg)[0])
    G.check_device_error()
    specs = m.specs
    m.close()
    torch.cuda.empty_cache()

    ref = OracleModel(cfg, specs, threads=max(8, os.cpu_count() or 8))
    for pos, t in enumerate(prompt[:-1]):
        ref.step(t, pos, fp16_cache=True, head=False)
    feed, rels, match = prompt[-1], [], 0
    for i in range(N_NEW):
        y = ref.step(feed, N_PROMPT - 1 + i, fp16_cache=True)
        rels.append(rel(logits[i], y))
        match += int(O.argmax(y)[0] == toks[i])
        feed = toks[i]
    rate = match / N_NEW
    print("config 3, 28 layers: logits rel-L2 per step %s, token match %.2f, tokens %s"
          % (["%.2e" % r for r in rels], rate, toks))
    assert all(np.isfinite(lg).all() for lg in logits)
    assert max(rels) <= 1e-2
    assert rate == 1.0
