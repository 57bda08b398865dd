"""The attention softmax's FMA-pipe exponential (f2_exp2_poly in
csrc/kernels/sm100_ptx.cuh), restated on the CPU from the coefficients in the source:
x = j + f with j = round(x) through the 1.5 * 2^23 shifter, 2^f from the degree-4
polynomial in Horner form with each multiply-add rounded once to fp32 as the device's
fused multiply-add does (the fp32 product is exact in float64), 2^j added to the
exponent field. The
relative error must stay within the 2.7e-6 the source states, over the whole range
the softmax feeds it ([-125, 8]) and at the interval ends f = +-0.5."""
import os
import re

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _coefficients():
    src = open(os.path.join(ROOT, "clove_compute_b200", "csrc", "kernels", "sm100_ptx.cuh")).read()
    body = src[src.index("uint64_t f2_exp2_poly("):]
    body = body[:body.index("\n}\n")]
    # f2_pack(c, c) pairs, in source order: c4, c3, c2, c1, c0.
    vals = [float(m) for m in re.findall(r"f2_pack\(([0-9.e+-]+)f, \1f\)", body)]
    vals = [v for v in vals if 0.0 < v < 2.0]  # drop the shifter and -1 constants
    assert len(vals) == 5, vals
    return [np.float32(v) for v in vals]


def _exp2_poly(x):
    c4, c3, c2, c1, c0 = _coefficients()
    f32 = np.float32
    x = np.maximum(x.astype(np.float32), f32(-125.0))
    t = (x + f32(12582912.0)).astype(np.float32)
    j = (t - f32(12582912.0)).astype(np.float32)
    f = (x - j).astype(np.float32)
    def fma(a, b, c):  # a * b + c with one rounding to fp32
        return (a.astype(np.float64) * b.astype(np.float64) + np.float64(c)).astype(np.float32)

    q = fma(f, np.full_like(f, c4), c3)
    for c in (c2, c1, c0):
        q = fma(q, f, c)
    bits = q.view(np.uint32) + (t.view(np.uint32) << np.uint32(23))
    return bits.view(np.float32)


def test_exp2_polynomial_bound_from_source_coefficients():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.uniform(-125.0, 8.0, 2_000_000), np.arange(-125.0, 8.5, 0.5),
                        np.array([-1e-7, 0.0, 1e-7])]).astype(np.float32)
    y = _exp2_poly(x).astype(np.float64)
    rel = np.abs(y / np.exp2(x.astype(np.float64)) - 1.0)
    assert rel.max() <= 2.7e-6, (rel.max(), x[np.argmax(rel)])
    low = _exp2_poly(np.array([-126.0, -1e4], dtype=np.float32)).astype(np.float64)
    assert np.all(np.abs(low / 2.0 ** -125 - 1.0) <= 2.7e-6)
