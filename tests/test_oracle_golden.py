"""Pin the C restatement (oracle/orc.c) against golden vectors produced by the
reference's own CPU code (tests/golden/make_golden.py).  Bit-exact throughout:
the restatement follows the reference's operation order exactly."""
import ctypes as C
import hashlib

import numpy as np
import pytest

import oracle as O


def same_bits(a, b):
    a = np.ascontiguousarray(a, np.float32).view(np.uint32)
    b = np.ascontiguousarray(b, np.float32).view(np.uint32)
    return a.shape == b.shape and np.array_equal(a, b)


def sha(a):
    return np.frombuffer(hashlib.sha256(np.ascontiguousarray(a).tobytes()).digest(), np.uint8)


def test_half_to_float_exhaustive(golden):
    out = np.array([O.orc.orc_half_to_float(int(h)) for h in golden["half_in"]], np.float32)
    assert same_bits(out, golden["half_out"])


@pytest.mark.parametrize("fmt,bs", [("q4k", 144), ("q6k", 210)])
def test_dequant_rows(golden, fmt, bs):
    w = golden[fmt + "_deq_w"]
    k = int(golden[fmt + "_deq_k"][0])
    rows = w.size // ((k // 256) * bs)
    assert same_bits(O.dequant(fmt, w, rows, k).ravel(), golden[fmt + "_deq_y"])


@pytest.mark.parametrize("fmt,k", [("q4k", 3584), ("q6k", 3584), ("q4k", 18944), ("q6k", 18944)])
def test_matvec_rows(golden, fmt, k):
    tag = "%s_mv_%d" % (fmt, k)
    rows, wseed, xseed, bseed = [int(v) for v in golden[tag + "_seeds"]]
    w = O.fill_weights(fmt, rows, k, wseed)
    x = O.normal_f32(k, xseed)
    bias = O.normal_f32(rows, bseed, 0.0, 0.02)
    # the fixture generators themselves are pinned by digest
    assert np.array_equal(sha(w), golden[tag + "_w_sha"])
    assert np.array_equal(sha(x), golden[tag + "_x_sha"])
    assert np.array_equal(sha(bias), golden[tag + "_bias_sha"])
    assert same_bits(O.matvec(fmt, w, rows, k, x), golden[tag + "_y"])
    assert same_bits(O.matvec(fmt, w, rows, k, x, bias), golden[tag + "_yb"])
    # the row-parallel form gives the same bits as the reference's serial one
    assert same_bits(O.matvec(fmt, w, rows, k, x, bias, threads=3), golden[tag + "_yb"])


@pytest.mark.parametrize("s", range(5))
def test_q6_conditioning_strata(golden, s):
    w, x = golden["q6cb_%d_w" % s], golden["q6cb_%d_x" % s]
    n = x.size
    rows = w.size // ((n // 256) * 210)
    assert same_bits(O.dequant("q6k", w, rows, n).ravel(), golden["q6cb_%d_deq" % s])
    assert same_bits(O.matvec("q6k", w, rows, n, x), golden["q6cb_%d_y" % s])


def test_rmsnorm_swiglu_add(golden):
    assert same_bits(O.rmsnorm(golden["rms_x"], golden["rms_g"], 1e-6), golden["rms_y"])
    assert same_bits(O.swiglu(golden["swiglu_g"], golden["swiglu_u"]), golden["swiglu_y"])
    assert same_bits(O.add(golden["swiglu_g"], golden["swiglu_u"]), golden["add_y"])


@pytest.mark.parametrize("pos", [0, 1, 255, 4095])
@pytest.mark.parametrize("heads", [28, 4])
def test_rope(golden, pos, heads):
    x = golden["rope_%d_%d_x" % (pos, heads)]
    assert same_bits(O.rope(x, heads, 128, pos, 1.0e6), golden["rope_%d_%d_y" % (pos, heads)])


@pytest.mark.parametrize("layer,pos", [(0, 0), (1, 17), (1, 63)])
def test_attention_cache(golden, layer, pos):
    max_ctx, layers, kvd = 64, 2, 4 * 128
    kc = O.normal_f32(layers * max_ctx * kvd, 0x31)
    vc = O.normal_f32(layers * max_ctx * kvd, 0x32)
    assert np.array_equal(sha(kc), golden["attn_kc_sha"]) and np.array_equal(sha(vc), golden["attn_vc_sha"])
    q = O.normal_f32(28 * 128, 0x33 + pos)
    out = O.attention_cache(q, kc, vc, layer, pos, max_ctx, 28, 4, 128)
    assert same_bits(out, golden["attn_%d_%d_y" % (layer, pos)])


def test_argmax(golden):
    for i in range(5):
        if i < 4:
            x = golden["argmax_%d_x" % i]
        else:
            x = O.normal_f32(152064, 0x41)
            assert np.array_equal(sha(x), golden["argmax_4_x"])
        idx, fin = O.argmax(x)
        assert [idx, int(fin)] == list(golden["argmax_%d_y" % i])


def test_exec148_known_answers(golden):
    # the EXEC148 canonical tuple of each Q4_K block equals the decoded
    # (d, dmin, 8 x (sc, mn), 256 codes) of that block
    src, tup = golden["exec148_src"], golden["exec148_tuple"]
    for i in range(src.size // 144):
        b = src[i * 144:(i + 1) * 144]
        t = tup[i * 276:(i + 1) * 276]
        assert list(t[:4]) == list(b[:4])
        for j in range(8):
            sc, mn = C.c_uint8(0), C.c_uint8(0)
            O.orc.orc_q4k_scale_min.argtypes = [np.ctypeslib.ndpointer(np.uint8), C.c_int,
                                                 C.POINTER(C.c_uint8), C.POINTER(C.c_uint8)]
            O.orc.orc_q4k_scale_min(np.ascontiguousarray(b), j, C.byref(sc), C.byref(mn))
            assert (t[4 + 2 * j], t[5 + 2 * j]) == (sc.value, mn.value)
    assert bytes(golden["sha256_abc"]).hex() == \
        "ba7816bf8f01cfea414140de5dae2223b00361a396177a9cb410ff61f20015ad"


def test_reference_library_agrees_when_present():
    """Where the reference checkout exists, re-derive a few golden values live."""
    if O.ref is None:
        pytest.skip("reference CPU library not built here")
    w = O.fill_q6k(8, 3584, 99)
    x = O.normal_f32(3584, 98)
    y = np.empty(8, np.float32)
    O.ref.ref_matmul_q6(w, 3584, 8, 1, x, None, y)
    assert same_bits(O.matvec("q6k", w, 8, 3584, x), y)
