"""GGUF v3 files for the ArcLLM runtime: a writer for synthetic Qwen2 models
and a header reader.

The runtime's ``generate()`` consumes a GGUF file (``RunRequest.model_path``).
No checkpoint can be downloaded here, so tests and benchmarks write synthetic
Qwen2-architecture files with this module: the same metadata keys and tensor
names as a llama.cpp Qwen2 conversion (``qwen2.block_count``,
``blk.N.attn_q.weight`` ...), weights supplied by the caller as raw packed
bytes (Q4_K / Q6_K super-blocks, fp32 norms and biases, fp16 or Q4_K
embedding).

Layout written: magic ``GGUF``, version 3, tensor count, metadata count, the
metadata key/values, the tensor infos (name, dims with the row length first,
ggml type, offset relative to the data section), padding to ``alignment``,
then each tensor's bytes at an ``alignment`` multiple.
"""
import struct

GGUF_U32, GGUF_F32, GGUF_STRING, GGUF_ARRAY, GGUF_U64 = 4, 6, 8, 9, 10

# synthetic-model slot name (arcllm_b200.synthetic) -> GGUF tensor name suffix
LAYER_NAMES = {
    "attn_norm": "attn_norm.weight", "wq": "attn_q.weight", "bq": "attn_q.bias", "wk": "attn_k.weight",
    "bk": "attn_k.bias", "wv": "attn_v.weight", "bv": "attn_v.bias", "wo": "attn_output.weight",
    "ffn_norm": "ffn_norm.weight", "w_gate": "ffn_gate.weight", "w_up": "ffn_up.weight",
    "w_down": "ffn_down.weight",
}
ENDPOINT_NAMES = {"tok_embd": "token_embd.weight", "output_norm": "output_norm.weight", "output": "output.weight"}


def gguf_name(spec_name):
    """'blk.3.wq' -> 'blk.3.attn_q.weight'; 'output' -> 'output.weight'"""
    if spec_name in ENDPOINT_NAMES:
        return ENDPOINT_NAMES[spec_name]
    blk, l, slot = spec_name.split(".", 2)
    return "%s.%s.%s" % (blk, l, LAYER_NAMES[slot])


def _str(s):
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _kv(key, typ, value):
    out = _str(key) + struct.pack("<I", typ)
    if typ == GGUF_U32:
        return out + struct.pack("<I", value)
    if typ == GGUF_F32:
        return out + struct.pack("<f", value)
    if typ == GGUF_U64:
        return out + struct.pack("<Q", value)
    if typ == GGUF_STRING:
        return out + _str(value)
    raise ValueError("unsupported metadata type %r" % typ)


def qwen2_metadata(cfg, alignment=32):
    """Metadata of a llama.cpp Qwen2 conversion for the model config dict used
    by arcllm_b200.synthetic (n_layers, hidden, n_heads, n_kv_heads, ffn,
    max_ctx, rms_eps, rope_theta)."""
    return [
        ("general.architecture", GGUF_STRING, "qwen2"),
        ("general.name", GGUF_STRING, "synthetic-qwen2"),
        ("general.alignment", GGUF_U32, alignment),
        ("qwen2.block_count", GGUF_U32, cfg["n_layers"]),
        ("qwen2.context_length", GGUF_U32, cfg.get("max_ctx", 4096)),
        ("qwen2.embedding_length", GGUF_U32, cfg["hidden"]),
        ("qwen2.feed_forward_length", GGUF_U32, cfg["ffn"]),
        ("qwen2.attention.head_count", GGUF_U32, cfg["n_heads"]),
        ("qwen2.attention.head_count_kv", GGUF_U32, cfg["n_kv_heads"]),
        ("qwen2.rope.freq_base", GGUF_F32, cfg["rope_theta"]),
        ("qwen2.attention.layer_norm_rms_epsilon", GGUF_F32, cfg["rms_eps"]),
    ]


def write_gguf(path, metadata, tensors, alignment=32):
    """metadata: [(key, type, value)]; tensors: [(name, ggml_type, dims, data)]
    where dims lists the row length first and data is a bytes-like object of
    exactly the tensor's packed bytes.  Returns {name: absolute file offset}."""
    head = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(metadata))
    head += b"".join(_kv(k, t, v) for k, t, v in metadata)
    rel, off = [], 0
    for name, typ, dims, data in tensors:
        off = (off + alignment - 1) // alignment * alignment
        rel.append(off)
        head += _str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", typ, off)
        off += len(memoryview(data).cast("B"))
    data_off = (len(head) + alignment - 1) // alignment * alignment
    where = {}
    with open(path, "wb") as f:
        f.write(head)
        f.write(b"\0" * (data_off - len(head)))
        pos = data_off
        for (name, typ, dims, data), r in zip(tensors, rel):
            f.write(b"\0" * (data_off + r - pos))
            mv = memoryview(data).cast("B")
            f.write(mv)
            where[name] = data_off + r
            pos = data_off + r + len(mv)
    return where


def read_gguf_header(path):
    """(version, metadata {key: value}, tensors [(name, dims, type, offset)], data_offset)
    for files written by write_gguf (scalar and string metadata only)."""
    with open(path, "rb") as f:
        buf = f.read()
    pos = 0

    def take(fmt):
        nonlocal pos
        v = struct.unpack_from(fmt, buf, pos)
        pos += struct.calcsize(fmt)
        return v if len(v) > 1 else v[0]

    def string():
        nonlocal pos
        n = take("<Q")
        s = buf[pos:pos + n].decode("utf-8")
        pos += n
        return s

    if buf[:4] != b"GGUF":
        raise ValueError("not a GGUF file")
    pos = 4
    version, n_t, n_kv = take("<I"), take("<Q"), take("<Q")
    meta = {}
    for _ in range(n_kv):
        k, t = string(), take("<I")
        meta[k] = {GGUF_U32: lambda: take("<I"), GGUF_F32: lambda: take("<f"), GGUF_U64: lambda: take("<Q"),
                   GGUF_STRING: string}[t]()
    ts = []
    for _ in range(n_t):
        name = string()
        nd = take("<I")
        dims = [take("<Q") for _ in range(nd)]
        typ, off = take("<I"), take("<Q")
        ts.append((name, dims, typ, off))
    align = meta.get("general.alignment", 32)
    return version, meta, ts, (pos + align - 1) // align * align
