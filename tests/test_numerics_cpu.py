"""Numeric schemes of the tensor-core kernels, checked on the CPU.

The batched-prefill attention feeds q to fp16 MMAs as two halves, q*scale =
hi + lo with hi = fp16(q*scale) and lo = fp16(q*scale - hi); the cache keys are
fp16 already and the MMA forms exact products accumulated in fp32.  The scores
then carry an error of about 2^-22 of sum |q k| -- far below what a bf16 or a
single fp16 operand would give, which matters for the near-one-hot attention of
the synthetic models (scores of 1e3 .. 1e4).  This restates that scheme in
numpy (fp32 accumulation in the kernel's k-chunk order) against float64.
"""
import numpy as np


def split_scores(q, k):
    """S[i, p] as the kernel forms it: per 16-wide k step, hi then lo products
    (exact in fp32 for fp16 x fp16), accumulated in fp32."""
    hi = q.astype(np.float16)
    lo = (q - hi.astype(np.float32)).astype(np.float16)
    kf = k.astype(np.float32)
    s = np.zeros((q.shape[0], k.shape[0]), np.float32)
    for c in range(0, q.shape[1], 16):
        s = s + hi[:, c:c + 16].astype(np.float32) @ kf[:, c:c + 16].T
        s = s + lo[:, c:c + 16].astype(np.float32) @ kf[:, c:c + 16].T
    return s


def test_prefill_attention_score_split_precision():
    rng = np.random.default_rng(7)
    d, scale = 128, 1.0 / np.sqrt(128.0)
    # keys with row norms in the synthetic models' range, queries of similar size
    k = (rng.standard_normal((64, d)) * 150.0).astype(np.float16)
    q = (rng.standard_normal((14, d)) * 150.0).astype(np.float32) * np.float32(scale)
    exact = q.astype(np.float64) @ k.astype(np.float64).T
    mag = np.abs(q.astype(np.float64)) @ np.abs(k.astype(np.float64)).T
    got = split_scores(q, k).astype(np.float64)
    assert np.abs(got - exact).max() <= 2.0 ** -19 * mag.max()
    # a single fp16 operand would be ~2^-11 off: the split is what keeps softmax sharp
    single = (q.astype(np.float16).astype(np.float64) @ k.astype(np.float64).T)
    assert np.abs(single - exact).max() > 2.0 ** -14 * mag.max()


def test_prefill_attention_score_split_range_edges():
    """Where the hi + lo split holds: up to the fp16 maximum (65504) the scores
    keep the 2^-19 relative bound; past it hi overflows to inf, which the kernel
    reports through the device error word's range bit instead of returning NaN
    rows; for tiny |q * scale| the halves go subnormal and the error is bounded
    by the fp16 subnormal spacing (2^-24) times sum |k| rather than relatively."""
    rng = np.random.default_rng(11)
    d = 128
    k = (rng.standard_normal((32, d)) * 4.0).astype(np.float16)
    big = (rng.uniform(-1, 1, (4, d)) * 6.0e4).astype(np.float32)  # just inside the fp16 range
    exact = big.astype(np.float64) @ k.astype(np.float64).T
    mag = np.abs(big.astype(np.float64)) @ np.abs(k.astype(np.float64)).T
    assert np.abs(split_scores(big, k).astype(np.float64) - exact).max() <= 2.0 ** -19 * mag.max()
    over = np.full((1, d), 7.0e4, np.float32)  # past 65504: hi is inf -- the condition the kernel flags
    with np.errstate(over="ignore"):
        assert np.isinf(over.astype(np.float16)).all()
    tiny = (rng.standard_normal((4, d)) * 1e-6).astype(np.float32)
    exact = tiny.astype(np.float64) @ k.astype(np.float64).T
    err = np.abs(split_scores(tiny, k).astype(np.float64) - exact).max()
    assert err <= 2.0 ** -24 * np.abs(k.astype(np.float64)).sum(axis=1).max()
