"""Generate tests/golden/reference_golden.npz from the reference's OWN CPU code.

Runs in a container that has the ArcLLM checkout: oracle/build.py compiles
src/p8c_segmented_access_correctness.cpp, src/q6cb_fixture_generator.hpp and
src/q4_down_exec148_materializer.h in place into oracle/_ref/libref_cpu.so,
and this script records inputs + the reference's outputs.  The fixture file
lets the C restatement (oracle/orc.c) be pinned on machines without the
reference (the GPU box).  Usage:  python tests/golden/make_golden.py
"""
import ctypes as C
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle as O  # noqa: E402

OUT = os.path.join(HERE, "reference_golden.npz")


def digest(a):
    """sha256 of an array's bytes; inputs that the oracle's own generators can
    regenerate from a seed are stored as (seed, digest) to keep the file small."""
    import hashlib
    return np.frombuffer(hashlib.sha256(np.ascontiguousarray(a).tobytes()).digest(), np.uint8).copy()


def ref_rows(fn, w, rows, k, rb):
    y = np.empty(rows * k, np.float32)
    for r in range(rows):
        fn(w[r * rb:(r + 1) * rb], y[r * k:(r + 1) * k], k)
    return y


def main():
    R = O.ref
    if R is None:
        raise SystemExit("the reference CPU library is not available (needs the ArcLLM checkout)")
    g = {}
    rng = np.random.default_rng(20261201)

    # 1. fp16 decode, exhaustive
    h = np.arange(65536, dtype=np.uint16)
    g["half_in"] = h
    g["half_out"] = np.array([R.ref_half_to_float(int(v)) for v in h], np.float32)

    # 2. super-block dequant: synthetic fixture blocks + raw random bytes with
    #    hand-picked d/dmin (normal, subnormal, zero, negative) so every decode
    #    branch is exercised.  NaN/Inf d are excluded (matvec NaN payloads are
    #    not comparable); they are covered by half_in/half_out.
    for fmt, bs in (("q4k", 144), ("q6k", 210)):
        k, rows = 512, 12
        w_fix = O.fill_weights(fmt, rows, k, 0xA11CE)
        w_rnd = rng.integers(0, 256, size=rows * (k // 256) * bs, dtype=np.uint8)
        specials = [0x2800, 0x0001, 0x03FF, 0x0000, 0x8400, 0x3C00, 0xB800, 0x1400]
        for i in range(rows * (k // 256)):
            blk = w_rnd[i * bs:(i + 1) * bs]
            if fmt == "q4k":
                d, m = specials[i % 8], specials[(i + 3) % 8]
                blk[0:2] = [d & 255, d >> 8]
                blk[2:4] = [m & 255, m >> 8]
            else:
                d = specials[i % 8]
                blk[208:210] = [d & 255, d >> 8]
        w = np.concatenate([w_fix, w_rnd])
        rb = (k // 256) * bs
        fn = R.ref_q4k_dequant_row if fmt == "q4k" else R.ref_q6k_dequant_row
        g[fmt + "_deq_w"] = w
        g[fmt + "_deq_k"] = np.array([k])
        g[fmt + "_deq_y"] = ref_rows(fn, w, 2 * rows, k, rb)

    # 3. matvec (reference matmul_q4_cpu / matmul_q6_cpu), with and without bias
    for fmt, k, rows in (("q4k", 3584, 24), ("q6k", 3584, 24), ("q4k", 18944, 4), ("q6k", 18944, 4)):
        w = O.fill_weights(fmt, rows, k, 0xB0B + k + rows)
        x = O.normal_f32(k, 0x5EED + k)
        bias = O.normal_f32(rows, 0xB1A5, 0.0, 0.02)
        y = np.empty(rows, np.float32)
        yb = np.empty(rows, np.float32)
        fn = R.ref_matmul_q4 if fmt == "q4k" else R.ref_matmul_q6
        fn(w, k, rows, 1, x, None, y)
        fn(w, k, rows, 1, x, bias.ctypes.data_as(C.c_void_p), yb)
        tag = "%s_mv_%d" % (fmt, k)
        g[tag + "_seeds"] = np.array([rows, 0xB0B + k + rows, 0x5EED + k, 0xB1A5], np.uint64)
        g[tag + "_w_sha"], g[tag + "_x_sha"], g[tag + "_bias_sha"] = digest(w), digest(x), digest(bias)
        g[tag + "_y"], g[tag + "_yb"] = y, yb

    # 4. Q6_K conditioning strata (q6cb_fixture_generator.hpp) + reference matvec
    for s in range(5):
        n, rows = 512, 8
        nb = n // 256
        packed = np.empty(rows * nb * 210, np.uint8)
        x = np.empty(n, np.float32)
        ok = R.ref_q6cb_fixture(n, rows, 0x51CB0000 + s, s, packed, x)
        assert ok == 1
        y = np.empty(rows, np.float32)
        R.ref_matmul_q6(packed, n, rows, 1, x, None, y)
        g["q6cb_%d_w" % s], g["q6cb_%d_x" % s], g["q6cb_%d_y" % s] = packed, x, y
        g["q6cb_%d_deq" % s] = ref_rows(R.ref_q6k_dequant_row, packed, rows, n, nb * 210)

    # 5. rmsnorm (eps 1e-6), swiglu, add
    x = O.normal_f32(2 * 3584, 0x11)
    gam = O.normal_f32(3584, 0x12, 1.0, 0.1)
    y = np.empty_like(x)
    R.ref_rmsnorm(x, gam, 2, 3584, 1e-6, y)
    g["rms_x"], g["rms_g"], g["rms_y"] = x, gam, y
    a = O.normal_f32(18944, 0x13, 0.0, 3.0)
    b = O.normal_f32(18944, 0x14)
    y = np.empty_like(a)
    R.ref_swiglu(a, b, a.size, y)
    g["swiglu_g"], g["swiglu_u"], g["swiglu_y"] = a, b, y
    y = np.empty_like(a)
    R.ref_add(a, b, a.size, y)
    g["add_y"] = y

    # 6. RoPE on q (28 heads) and k (4 heads) at several positions, theta 1e6
    for pos in (0, 1, 255, 4095):
        for heads in (28, 4):
            x = O.normal_f32(heads * 128, 0x20 + pos + heads)
            y = x.copy()
            R.ref_rope(y, 1, heads, 128, pos, 1.0e6)
            g["rope_%d_%d_x" % (pos, heads)], g["rope_%d_%d_y" % (pos, heads)] = x, y

    # 7. cached GQA attention (28 q heads, 4 kv heads, dim 128) on a 2-layer fp32 cache
    max_ctx, layers, kvd = 64, 2, 4 * 128
    kc = O.normal_f32(layers * max_ctx * kvd, 0x31)
    vc = O.normal_f32(layers * max_ctx * kvd, 0x32)
    g["attn_kc_sha"], g["attn_vc_sha"] = digest(kc), digest(vc)
    for layer, pos in ((0, 0), (1, 17), (1, 63)):
        q = O.normal_f32(28 * 128, 0x33 + pos)
        out = np.empty(28 * 128, np.float32)
        R.ref_attention_cache(q, kc, vc, kc.size, layer, pos, max_ctx, 28, 4, 128, out)
        g["attn_%d_%d_y" % (layer, pos)] = out

    # 8. greedy argmax: ties keep the first index, non-finite flagged
    cases = [np.array([1, 3, 3, 2], np.float32), np.array([-5, -1, -1, -7], np.float32),
             np.array([0, np.nan, 4, 4], np.float32), np.array([np.inf, 1, 2], np.float32),
             O.normal_f32(152064, 0x41)]
    for i, c in enumerate(cases):
        fin = C.c_int(0)
        idx = R.ref_argmax(c, c.size, C.byref(fin))
        g["argmax_%d_x" % i] = c if c.size < 100 else digest(c)
        g["argmax_%d_y" % i] = np.array([idx, fin.value], np.int64)

    # 9. EXEC148 materializer known answers (src/q4_down_exec148_materializer.h)
    src = O.fill_q4k(1, 3584, 0xE148)
    nblk = src.size // 144
    exe = np.empty(nblk * 148, np.uint8)
    tup = np.empty(nblk * 276, np.uint8)
    for i in range(nblk):
        R.ref_exec148_materialize_block(src[i * 144:(i + 1) * 144], exe[i * 148:(i + 1) * 148])
        R.ref_exec148_source_tuple(src[i * 144:(i + 1) * 144], tup[i * 276:(i + 1) * 276])
    g["exec148_src"], g["exec148_exe"], g["exec148_tuple"] = src, exe, tup
    dig = np.empty(32, np.uint8)
    R.ref_sha256(np.frombuffer(b"abc", np.uint8).copy(), 3, dig)
    g["sha256_abc"] = dig

    np.savez_compressed(OUT, **g)
    print("wrote", OUT, os.path.getsize(OUT), "bytes,", len(g), "arrays")


if __name__ == "__main__":
    main()
