"""Synthetic Qwen2 GGUF files for the runtime tests (TEST INFRASTRUCTURE).

Tensor bytes come from the oracle's fixture generators with the seeds of
arcllm_b200.synthetic.tensor_specs, so a file written here holds exactly the
weights SyntheticModel fills on the device for the same config and seed.
"""
import numpy as np

import oracle as O
from arcllm_b200 import GGML_Q4_K
from arcllm_b200.gguf import gguf_name, qwen2_metadata, write_gguf
from arcllm_b200.synthetic import tensor_specs


def tensor_data(s):
    if s["kind"] == "quant":
        fmt = "q4k" if s["type"] == GGML_Q4_K else "q6k"
        return O.fill_weights(fmt, s["rows"], s["cols"], s["seed"])
    if s["kind"] == "normal16":
        return np.ascontiguousarray(O.normal_f16(s["rows"] * s["cols"], s["seed"], s["mu"], s["sigma"]))
    return O.normal_f32(s["rows"] * s["cols"], s["seed"], s["mu"], s["sigma"])


def write_synthetic_gguf(path, cfg, types=None, seed=0xA2C11, drop=(), override=None):
    """Write the synthetic model as GGUF.  `drop` omits tensors (GGUF names);
    `override` maps GGUF names to (ggml_type, dims, data) replacements."""
    specs = tensor_specs(cfg, types, seed)
    order = ["tok_embd"] + [n for n in specs if n.startswith("blk.")] + ["output_norm", "output"]
    tensors = []
    for n in order:
        s, g = specs[n], gguf_name(n)
        if g in drop:
            continue
        if override and g in override:
            typ, dims, data = override[g]
        else:
            dims = [s["cols"]] if s["rows"] == 1 else [s["cols"], s["rows"]]
            typ, data = s["type"], tensor_data(s)
        tensors.append((g, typ, dims, data))
    write_gguf(path, qwen2_metadata(cfg), tensors)
    return specs
