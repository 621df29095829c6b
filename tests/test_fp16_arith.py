"""The identities behind the tail kernel's half-precision adds and multiplies.

The reference rounds fp16 sums the fp32 way (both operands widened, added in fp32,
the result rounded to fp16), and the tail computes those same sums with half-precision
adds (which return the exact sum rounded once to fp16). They agree when
RN16(RN32(a + b)) == RN16(a + b) for all fp16 a, b, and likewise for a * 0.5. Checked
here on the CPU: every finite fp16 value against a sample of second operands (zeros,
subnormals, the extremes and random values), with the exact sum taken in float64
(exact for any two fp16 values: at most 11 + 40 significant bits).
"""
import numpy as np


def _all_finite_fp16():
    bits = np.arange(1 << 16, dtype=np.uint16)
    v = bits.view(np.float16)
    return v[np.isfinite(v)]


def test_fp32_rounded_fp16_sum_equals_exact_rounded_sum():
    a = _all_finite_fp16()
    rng = np.random.default_rng(0)
    edge = np.array([0.0, -0.0, 2.0 ** -24, -(2.0 ** -24), 2.0 ** -14, 65504.0, -65504.0, 1.0, -1.0,
                     1.0 + 2.0 ** -10, 2048.0, 2.0 ** -13], dtype=np.float16)
    b = np.concatenate([edge, rng.choice(a, 400, replace=False)])
    for bv in b:
        with np.errstate(over="ignore", invalid="ignore"):     # sums past 65504 become inf both ways
            via32 = (a.astype(np.float32) + np.float32(bv)).astype(np.float16)
            exact = (a.astype(np.float64) + np.float64(bv)).astype(np.float16)
        same = (via32 == exact) | (np.isnan(via32) & np.isnan(exact))
        # signed zeros compare equal; the kernels' ordering treats -0 and +0 alike as well
        assert same.all(), (float(bv), a[~same][:5])


def test_fp32_rounded_half_product_equals_exact():
    a = _all_finite_fp16()
    via32 = (a.astype(np.float32) * np.float32(0.5)).astype(np.float16)
    exact = (a.astype(np.float64) * 0.5).astype(np.float16)
    assert np.array_equal(via32.view(np.uint16), exact.view(np.uint16))
