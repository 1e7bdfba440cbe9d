"""Synthetic Qwen2-family models generated directly in HBM.

There is no network and no checkpoint here, so benchmarks and tests use
random-init weights of the real architecture.  Every tensor is filled on the
device by the library's counter-based fixture generators
(``arcllm_cuda_fill_*``), one splitmix64 stream per tensor, so any tensor can
be regenerated bit-for-bit elsewhere (the CPU test oracle does exactly that).

Field distributions (the benchmark's decode workload): Q4_K super-blocks with
d ~ U[1e-3,4e-3), dmin ~ U[0,2e-3), 6-bit scales/mins and 4-bit codes uniform;
Q6_K with uniform 6-bit codes, int8 scales in [-32,31], d ~ U[1e-3,4e-3);
RMSNorm weights ~ N(1, 0.1); QKV biases ~ N(0, 0.02); fp16 embedding ~ N(0, 0.02)
("normal" = Irwin-Hall sum of four 16-bit uniforms scaled to unit variance).
"""
import ctypes as C

from . import (GGML_F16, GGML_F32, GGML_Q4_K, GGML_Q6_K, GenStats, Layer, ModelConfig, call, lib, row_bytes)

QWEN25_7B = dict(n_layers=28, hidden=3584, n_heads=28, n_kv_heads=4, head_dim=128, ffn=18944, vocab=152064,
                 max_ctx=4096, rms_eps=1e-6, rope_theta=1.0e6)

# per-layer tensor slots (seed index = 16*layer + slot), endpoints after the layers
LAYER_SLOTS = ["attn_norm", "wq", "bq", "wk", "bk", "wv", "bv", "wo", "ffn_norm", "w_gate", "w_up", "w_down"]
ENDPOINT_SLOTS = ["tok_embd", "output_norm", "output"]

DEFAULT_TYPES = dict(wq=GGML_Q4_K, wk=GGML_Q4_K, wv=GGML_Q6_K, wo=GGML_Q4_K, w_gate=GGML_Q4_K, w_up=GGML_Q4_K,
                     w_down=GGML_Q6_K, output=GGML_Q6_K, tok_embd=GGML_F16)

_MASK = (1 << 64) - 1


def splitmix64_at(seed, n):
    """element n of the splitmix64 sequence of `seed` (same as the library)"""
    z = (seed + (n + 1) * 0x9E3779B97F4A7C15) & _MASK
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _MASK
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _MASK
    return z ^ (z >> 31)


def tensor_specs(cfg, types=None, seed=0xA2C11):
    """name -> dict(kind, type, rows, cols, seed, mu, sigma) for every tensor."""
    t = dict(DEFAULT_TYPES)
    t.update(types or {})
    H, F, V = cfg["hidden"], cfg["ffn"], cfg["vocab"]
    KV = cfg["n_kv_heads"] * cfg["head_dim"]
    L = cfg["n_layers"]
    specs = {}

    def add(name, idx, kind, typ, rows, cols, mu=0.0, sigma=0.0):
        specs[name] = dict(kind=kind, type=typ, rows=rows, cols=cols, seed=splitmix64_at(seed, idx), mu=mu,
                           sigma=sigma)

    for l in range(L):
        b = 16 * l
        p = "blk.%d." % l
        add(p + "attn_norm", b + 0, "normal", GGML_F32, 1, H, 1.0, 0.1)
        add(p + "wq", b + 1, "quant", t["wq"], H, H)
        add(p + "bq", b + 2, "normal", GGML_F32, 1, H, 0.0, 0.02)
        add(p + "wk", b + 3, "quant", t["wk"], KV, H)
        add(p + "bk", b + 4, "normal", GGML_F32, 1, KV, 0.0, 0.02)
        add(p + "wv", b + 5, "quant", t["wv"], KV, H)
        add(p + "bv", b + 6, "normal", GGML_F32, 1, KV, 0.0, 0.02)
        add(p + "wo", b + 7, "quant", t["wo"], H, H)
        add(p + "ffn_norm", b + 8, "normal", GGML_F32, 1, H, 1.0, 0.1)
        add(p + "w_gate", b + 9, "quant", t["w_gate"], F, H)
        add(p + "w_up", b + 10, "quant", t["w_up"], F, H)
        add(p + "w_down", b + 11, "quant", t["w_down"], H, F)
    e = 16 * L
    if t["tok_embd"] == GGML_F16:
        add("tok_embd", e + 0, "normal16", GGML_F16, V, H, 0.0, 0.02)
    else:
        add("tok_embd", e + 0, "quant", t["tok_embd"], V, H)
    add("output_norm", e + 1, "normal", GGML_F32, 1, H, 1.0, 0.1)
    add("output", e + 2, "quant", t["output"], V, H)
    return specs


def tensor_bytes(s):
    if s["kind"] == "quant":
        return s["rows"] * row_bytes(s["type"], s["cols"])
    if s["kind"] == "normal16":
        return 2 * s["rows"] * s["cols"]
    return 4 * s["rows"] * s["cols"]


class SyntheticModel:
    """A synthetic model resident on one GPU, wired into the C-ABI model."""

    def __init__(self, cfg=None, types=None, seed=0xA2C11, device=None, torch=None):
        """device: the CUDA device index (default: the current device, the one
        the library launches on -- tensors elsewhere would be another GPU's
        memory to the kernels)."""
        if torch is None:
            import torch
        self.torch = torch
        self.cfg = dict(QWEN25_7B if cfg is None else cfg)
        self.specs = tensor_specs(self.cfg, types, seed)
        if device is None:
            device = torch.cuda.current_device()
        elif device != torch.cuda.current_device():
            raise ValueError("SyntheticModel: device %d is not the current device %d" %
                             (device, torch.cuda.current_device()))
        self.dev = torch.device("cuda", device)
        L = lib()
        self.L = L
        self.stream = C.c_void_p(torch.cuda.current_stream(self.dev).cuda_stream)
        offs, off = {}, 0
        for name, s in self.specs.items():
            offs[name] = off
            off = (off + tensor_bytes(s) + 16 + 255) // 256 * 256
        self.weight_bytes = sum(tensor_bytes(s) for s in self.specs.values())
        self.arena = torch.empty(off, dtype=torch.uint8, device=self.dev)
        base = self.arena.data_ptr()
        self.ptr = {n: base + o for n, o in offs.items()}
        for name, s in self.specs.items():
            p = C.c_void_p(self.ptr[name])
            if s["kind"] == "quant":
                nblk = s["rows"] * (s["cols"] // 256)
                call("arcllm_cuda_fill_q4k" if s["type"] == GGML_Q4_K else "arcllm_cuda_fill_q6k", p, 0, nblk,
                     s["seed"], self.stream)
            elif s["kind"] == "normal16":
                call("arcllm_cuda_fill_normal_f16", p, 0, s["rows"] * s["cols"], s["seed"], C.c_float(s["mu"]),
                     C.c_float(s["sigma"]), self.stream)
            else:
                call("arcllm_cuda_fill_normal_f32", p, 0, s["rows"] * s["cols"], s["seed"], C.c_float(s["mu"]),
                     C.c_float(s["sigma"]), self.stream)
        c = self.cfg
        mc = ModelConfig(c["n_layers"], c["hidden"], c["n_heads"], c["n_kv_heads"], c["head_dim"], c["ffn"],
                         c["vocab"], c["max_ctx"], c["rms_eps"], c["rope_theta"])
        h = C.c_void_p()
        call("arcllm_cuda_model_create", C.byref(mc), C.byref(h))
        self.h = h
        for l in range(c["n_layers"]):
            p = "blk.%d." % l
            P = lambda n: C.c_void_p(self.ptr[p + n])  # noqa: E731
            T = lambda n: self.specs[p + n]["type"]  # noqa: E731
            lay = Layer(P("attn_norm"), P("wq"), P("bq"), T("wq"), P("wk"), P("bk"), T("wk"), P("wv"), P("bv"),
                        T("wv"), P("wo"), T("wo"), P("ffn_norm"), P("w_gate"), P("w_up"), T("w_gate"), P("w_down"),
                        T("w_down"))
            call("arcllm_cuda_model_set_layer", h, l, C.byref(lay))
        call("arcllm_cuda_model_set_endpoints", h, C.c_void_p(self.ptr["tok_embd"]), self.specs["tok_embd"]["type"],
             C.c_void_p(self.ptr["output_norm"]), C.c_void_p(self.ptr["output"]), self.specs["output"]["type"])

    # ---- generation ------------------------------------------------------
    def generate(self, prompt, max_new):
        n = len(prompt)
        pa = (C.c_uint32 * n)(*prompt)
        out = (C.c_uint32 * max_new)()
        st = GenStats()
        call("arcllm_cuda_model_generate", self.h, pa, n, max_new, out, C.byref(st), self.stream)
        return list(out), st

    def set_prefill_mode(self, mode):
        """1: batched tensor-core prefill (default); 0: token by token"""
        call("arcllm_cuda_model_set_prefill_mode", self.h, int(mode))

    def kv_cache(self, layer, n_pos):
        """fp16 K and V cache rows [n_pos][kv_dim] of one layer (numpy)"""
        import numpy as np
        c = self.cfg
        kv = c["n_kv_heads"] * c["head_dim"]
        kp, vp = C.c_void_p(), C.c_void_p()
        call("arcllm_cuda_model_kv_cache", self.h, C.byref(kp), C.byref(vp))
        out = []
        for p in (kp, vp):
            a = np.empty((n_pos, kv), np.float16)
            src = C.c_void_p(p.value + 2 * layer * c["max_ctx"] * kv)
            call("arcllm_cuda_memcpy_d2h", a.ctypes.data_as(C.c_void_p), src, a.nbytes, self.stream)
            out.append(a)
        call("arcllm_cuda_stream_synchronize", self.stream)
        return out

    def begin(self, prompt, max_new):
        pa = (C.c_uint32 * len(prompt))(*prompt)
        call("arcllm_cuda_model_begin", self.h, pa, len(prompt), max_new, self.stream)

    def set_tensor_parallel(self, ptrs, n_ranks, rank, timeout_us=2000000):
        """Shard the FFN and LM head over n_ranks (ptrs: ExchangeBuffers.ptrs
        with max_words from tp_exchange_words); n_ranks 1 turns it off."""
        call("arcllm_cuda_model_set_tensor_parallel", self.h, ptrs, n_ranks, rank, timeout_us)

    def tp_exchange_words(self, n_ranks):
        c = self.cfg
        mc = ModelConfig(c["n_layers"], c["hidden"], c["n_heads"], c["n_kv_heads"], c["head_dim"], c["ffn"],
                         c["vocab"], c["max_ctx"], c["rms_eps"], c["rope_theta"])
        out = C.c_uint32(0)
        call("arcllm_cuda_model_tp_exchange_words", C.byref(mc), n_ranks, C.byref(out))
        return out.value

    def prefill(self):
        """after begin(): consume the prompt but its last token as generate() does"""
        call("arcllm_cuda_model_prefill", self.h, self.stream)

    def step(self, with_head=True, use_graph=True):
        call("arcllm_cuda_model_step", self.h, 1 if with_head else 0, 1 if use_graph else 0, self.stream)

    def logits(self):
        """copy of the last logits (numpy)"""
        import numpy as np
        p = C.c_void_p()
        call("arcllm_cuda_model_logits", self.h, C.byref(p))
        out = np.empty(self.cfg["vocab"], np.float32)
        call("arcllm_cuda_memcpy_d2h", out.ctypes.data_as(C.c_void_p), p, out.nbytes, self.stream)
        call("arcllm_cuda_stream_synchronize", self.stream)
        return out

    def bytes_per_token(self):
        """algorithmic bytes read per decode token: every weight except the
        embedding table (one row of it), plus the embedding row"""
        emb = self.specs["tok_embd"]
        return self.weight_bytes - tensor_bytes(emb) + tensor_bytes(dict(emb, rows=1))

    def close(self):
        if self.h:
            call("arcllm_cuda_model_destroy", self.h)
            self.h = None
        self.arena = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
