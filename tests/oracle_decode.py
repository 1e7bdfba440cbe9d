"""CPU oracle for end-to-end greedy decode (TEST INFRASTRUCTURE ONLY).

Regenerates a synthetic model's tensors with the oracle's own fixture
generators (bit-identical to the device fill) and runs the reference's decode
algorithm layer by layer with the reference's CPU functions restated in
oracle/orc.c: RMSNorm, matmul_q4/q6 (+bias), RoPE, fp32 KV cache,
attention_cache_cpu, SwiGLU, residual adds, output norm, LM head, argmax --
the order of src/arcllm_v1_runtime.cpp:371-421.
"""
import numpy as np

import oracle as O
from arcllm_b200 import GGML_F16, GGML_Q4_K


class OracleModel:
    def __init__(self, cfg, specs, threads=8):
        from concurrent.futures import ThreadPoolExecutor
        self.cfg, self.specs, self.threads = cfg, specs, threads
        self.w = {}

        def make(item):  # the C fill routines release the GIL: tensors fill in parallel
            name, s = item
            if s["kind"] == "quant":
                fmt = "q4k" if s["type"] == GGML_Q4_K else "q6k"
                return name, (fmt, O.fill_weights(fmt, s["rows"], s["cols"], s["seed"]))
            if s["kind"] == "normal16":
                return name, ("f16", None)  # rows generated on demand
            return name, ("f32", O.normal_f32(s["rows"] * s["cols"], s["seed"], s["mu"], s["sigma"]))

        with ThreadPoolExecutor(max(1, threads)) as ex:
            self.w = dict(ex.map(make, specs.items()))
        L, C_, KV = cfg["n_layers"], cfg["max_ctx"], cfg["n_kv_heads"] * cfg["head_dim"]
        self.kc = np.zeros(L * C_ * KV, np.float32)
        self.vc = np.zeros(L * C_ * KV, np.float32)

    def mv(self, name, x, bias=None):
        fmt, w = self.w[name]
        s = self.specs[name]
        b = None if bias is None else self.w[bias][1]
        return O.matvec(fmt, w, s["rows"], s["cols"], x, b, threads=self.threads)

    def embed(self, tok):
        s = self.specs["tok_embd"]
        H = self.cfg["hidden"]
        if s["type"] == GGML_F16:
            row = O.normal_f16(H, s["seed"], s["mu"], s["sigma"], begin=tok * H)
            return row.view(np.float16).astype(np.float32)
        fmt, w = self.w["tok_embd"]
        rb = (H // 256) * 144
        return O.dequant(fmt, w[tok * rb:(tok + 1) * rb], 1, H).ravel()

    def step(self, tok, pos, fp16_cache=False, head=True):
        """Hidden state of token `tok` at position `pos` through every layer
        (its K/V rows land in the cache); the logits when `head`, else None."""
        c = self.cfg
        H, eps, th = c["hidden"], c["rms_eps"], c["rope_theta"]
        QH, KVH, D, MC = c["n_heads"], c["n_kv_heads"], c["head_dim"], c["max_ctx"]
        KV = KVH * D
        h = self.embed(tok)
        for l in range(c["n_layers"]):
            p = "blk.%d." % l
            xn = O.rmsnorm(h, self.w[p + "attn_norm"][1], eps)
            q = self.mv(p + "wq", xn, p + "bq")
            k = self.mv(p + "wk", xn, p + "bk")
            v = self.mv(p + "wv", xn, p + "bv")
            q = O.rope(q, QH, D, pos, th)
            k = O.rope(k, KVH, D, pos, th)
            if fp16_cache:
                k = k.astype(np.float16).astype(np.float32)
                v = v.astype(np.float16).astype(np.float32)
            base = (l * MC + pos) * KV
            self.kc[base:base + KV] = k
            self.vc[base:base + KV] = v
            a = O.attention_cache(q, self.kc, self.vc, l, pos, MC, QH, KVH, D)
            h1 = O.add(h, self.mv(p + "wo", a))
            xn2 = O.rmsnorm(h1, self.w[p + "ffn_norm"][1], eps)
            s = O.swiglu(self.mv(p + "w_gate", xn2), self.mv(p + "w_up", xn2))
            h = O.add(h1, self.mv(p + "w_down", s))
        if not head:
            return None
        xn = O.rmsnorm(h, self.w["output_norm"][1], eps)
        return self.mv("output", xn)
