"""CPU check of the prefill kernel's FMA-pipe exponential (ex2_poly in
vulcan_b200/csrc/vk_prefill_tc.cu): the same float32 steps restated in numpy
with the coefficients read from the source, compared with exp2 in float64.

Bound: relative error <= 1e-4 (half an fp16 ulp is 2.4e-4) for x in [-125, 8]
(P's exponent range under the kernel's lazy rescale, where fp16 still has
values); at and below the clamp (-126, -inf) the result is below 2e-38, which
rounds to fp16 zero."""
import os
import re

import numpy as np

SRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "vulcan_b200", "csrc",
                   "vk_prefill_tc.cu")


def _coeffs():
    text = open(SRC).read()
    body = text[text.index("float ex2_poly(float x)"):]
    body = body[:body.index("\n}\n")]
    nums = [float(x) for x in re.findall(r"(-?\d+\.\d+)f", body)]
    # kRound, clamp, then the Horner coefficients c3, c2, c1, c0
    return np.float32(nums[0]), np.float32(nums[1]), [np.float32(c) for c in nums[2:6]]


def ex2_poly(x):
    k_round, clamp, (c3, c2, c1, c0) = _coeffs()
    x = np.maximum(x.astype(np.float32), np.float32(clamp))
    t = (x + k_round).astype(np.float32)
    f = (x - (t - k_round).astype(np.float32)).astype(np.float32)
    p = np.float32(c3) * f + c2
    p = (p * f + c1).astype(np.float32)
    p = (p * f + c0).astype(np.float32)
    bits = p.view(np.int32) + (t.view(np.int32) << np.int32(23))
    return bits.astype(np.int32).view(np.float32)


def test_coefficients_parsed():
    k_round, clamp, c = _coeffs()
    assert k_round == np.float32(12582912.0) and clamp == np.float32(-126.0)
    assert len(c) == 4 and abs(float(c[3]) - 1.0) < 1e-3


def test_relative_error_bound():
    x = np.concatenate([np.linspace(-125.0, 8.0, 200001), np.arange(-125, 9, dtype=np.float64),
                        np.arange(-125, 8) + 0.5]).astype(np.float32)
    got = ex2_poly(x).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    rel = np.abs(got - want) / want
    assert rel.max() < 1e-4, rel.max()


def test_minus_infinity_rounds_to_fp16_zero():
    v = ex2_poly(np.array([-np.inf, -1000.0, -200.0, -126.0], np.float32))
    assert np.all(v >= 0) and np.all(v < 2e-38) and np.all(v.astype(np.float16) == 0)
