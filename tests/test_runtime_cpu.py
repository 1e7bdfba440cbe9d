"""C++ host runtime without a GPU: GGUF writing/reading, the request and model
checks of generate() (same messages and exit code 2 as the reference CLI,
src/arcllm_v1_runtime_cli.cpp:98-101 and src/arcllm_v1_runtime.cpp:153-252),
and the Q4CudaBackend status semantics."""
import json
import os
import subprocess

import numpy as np
import pytest

from arcllm_b200.gguf import read_gguf_header, write_gguf, GGUF_U32
from gguf_util import write_synthetic_gguf

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "arcllm_b200")
CLI = os.path.join(PKG, "arcllm_v1_runtime_cli")

TINY = dict(n_layers=2, hidden=256, n_heads=2, n_kv_heads=1, head_dim=128, ffn=512, vocab=512, max_ctx=64,
            rms_eps=1e-6, rope_theta=1.0e6)


def have_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="module", autouse=True)
def built():
    from arcllm_b200 import build as B
    B.build()
    B.build_runtime()


def cli(*args, **kw):
    r = subprocess.run([CLI] + [str(a) for a in args], capture_output=True, text=True, timeout=300, **kw)
    return r.returncode, r.stdout, r.stderr


def run_model(path, tokens="1,2,3", max_new=2, extra=()):
    return cli("--model", path, "--shader-dir", "unused", "--tokens", tokens, "--max-new", max_new, "--profile", 0,
               "--within-validated-domain", 0, *extra)


@pytest.fixture(scope="module")
def tiny_gguf(tmp_path_factory):
    p = str(tmp_path_factory.mktemp("gguf") / "tiny.gguf")
    write_synthetic_gguf(p, TINY)
    return p


def test_gguf_writer_roundtrip(tmp_path):
    p = str(tmp_path / "t.gguf")
    a = np.arange(256, dtype=np.float32)
    b = np.arange(144 * 2, dtype=np.uint8)
    where = write_gguf(p, [("general.alignment", GGUF_U32, 32), ("x.n", GGUF_U32, 7)],
                       [("a", 0, [256], a), ("b", 12, [256, 2], b)])
    ver, meta, ts, data_off = read_gguf_header(p)
    assert ver == 3 and meta["x.n"] == 7
    assert [t[0] for t in ts] == ["a", "b"] and ts[1][1] == [256, 2] and ts[1][2] == 12
    assert data_off % 32 == 0 and ts[1][3] % 32 == 0
    raw = open(p, "rb").read()
    assert raw[where["a"]:where["a"] + a.nbytes] == a.tobytes()
    assert raw[where["b"]:where["b"] + b.nbytes] == b.tobytes()
    assert where["a"] == data_off + ts[0][3]


def test_synthetic_gguf_census(tiny_gguf):
    _, meta, ts, _ = read_gguf_header(tiny_gguf)
    assert len(ts) == 12 * TINY["n_layers"] + 3
    assert meta["qwen2.block_count"] == 2 and meta["general.architecture"] == "qwen2"
    names = {t[0]: t for t in ts}
    assert names["blk.1.ffn_down.weight"][1] == [TINY["ffn"], TINY["hidden"]]
    assert names["output.weight"][1] == [TINY["hidden"], TINY["vocab"]]
    assert names["blk.0.attn_k.bias"][1] == [TINY["n_kv_heads"] * TINY["head_dim"]]


def test_cli_usage_errors():
    rc, out, err = cli()
    assert rc == 2 and "required: --model" in err
    rc, _, err = cli("--bogus")
    assert rc == 2 and "unknown argument" in err
    rc, _, err = cli("--model", "m", "--shader-dir", "s", "--tokens", "1,,2", "--max-new", "1", "--profile", "0",
                     "--within-validated-domain", "0")
    assert rc == 2 and "empty token" in err
    rc, _, err = cli("--model", "m", "--shader-dir", "s", "--tokens", "1", "--max-new", "1", "--profile", "2",
                     "--within-validated-domain", "0")
    assert rc == 2 and "--profile must be 0 or 1" in err


def test_request_checks(tiny_gguf, tmp_path):
    rc, _, err = run_model(tiny_gguf, max_new=0)
    assert rc == 2 and "max_new_tokens >= 1" in err
    rc, _, err = run_model(str(tmp_path / "missing.gguf"))
    assert rc == 2 and "cannot open GGUF" in err
    junk = tmp_path / "junk.gguf"
    junk.write_bytes(b"NOPE" + bytes(64))
    rc, _, err = run_model(str(junk))
    assert rc == 2 and "not a GGUF file" in err
    # limits of runtime.cpp:246-252
    rc, _, err = run_model(tiny_gguf, tokens=",".join(["1"] * 257))
    assert rc == 2 and "prefill token count exceeds" in err
    rc, _, err = run_model(tiny_gguf, tokens="1,2", max_new=4096)
    assert rc == 2 and "exceeds KV context limit" in err
    rc, _, err = run_model(tiny_gguf, tokens="1,%d" % TINY["vocab"])
    assert rc == 2 and "input token out of vocabulary" in err


def test_model_checks(tmp_path):
    p = str(tmp_path / "drop.gguf")
    write_synthetic_gguf(p, TINY, drop=("blk.1.attn_v.bias",))
    rc, _, err = run_model(p)
    assert rc == 2 and "census mismatch" in err
    # wrong type: an fp32 Q projection (the runtime runs Q4_K there)
    H = TINY["hidden"]
    p = str(tmp_path / "type.gguf")
    write_synthetic_gguf(p, TINY, override={"blk.0.attn_q.weight": (0, [H, H], np.zeros(H * H, np.float32))})
    rc, _, err = run_model(p)
    assert rc == 2 and "unsupported tensor type for blk.0.attn_q.weight" in err
    # wrong shape
    p = str(tmp_path / "shape.gguf")
    write_synthetic_gguf(p, TINY, override={"blk.1.ffn_norm.weight": (0, [H + 32], np.zeros(H + 32, np.float32))})
    rc, _, err = run_model(p)
    assert rc == 2 and "tensor shape mismatch: blk.1.ffn_norm.weight" in err
    # truncated payload -> TensorStore bounds invariant
    good = str(tmp_path / "good.gguf")
    write_synthetic_gguf(good, TINY)
    raw = open(good, "rb").read()
    cut = str(tmp_path / "cut.gguf")
    open(cut, "wb").write(raw[:len(raw) - 1000])
    rc, _, err = run_model(cut)
    assert rc == 2 and "TensorStore invariants failed" in err


@pytest.mark.skipif(have_gpu(), reason="checks the no-device path")
def test_valid_model_reaches_device_stage(tiny_gguf):
    """Every host-side check passes on a valid file; without a GPU the call
    then stops at the device query."""
    rc, out, err = run_model(tiny_gguf, tokens="5,6,7", max_new=3)
    assert rc == 2 and "found no CUDA device" in err, err


def build_test_program(tmp_path, name):
    exe = str(tmp_path / name)
    src = os.path.join(ROOT, "tests", "cpp", name + ".cpp")
    subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-I", os.path.join(ROOT, "include"), src, "-o", exe,
                    "-L", PKG, "-larcllm_runtime", "-larcllm_cuda", "-Wl,-rpath," + PKG], check=True)
    return exe


def test_q4_down_policy_decisions(tmp_path):
    r = subprocess.run([build_test_program(tmp_path, "q4_down_policy")], capture_output=True, text=True, timeout=60)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr


def test_q4_backend_status_semantics(tmp_path):
    exe = str(tmp_path / "q4_backend_status")
    src = os.path.join(ROOT, "tests", "cpp", "q4_backend_status.cpp")
    subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-I", os.path.join(ROOT, "include"), src, "-o", exe,
                    "-L", PKG, "-larcllm_runtime", "-larcllm_cuda", "-Wl,-rpath," + PKG], check=True)
    r = subprocess.run([exe, str(tmp_path), "gpu" if have_gpu() else "cpu"], capture_output=True, text=True,
                       timeout=120)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
