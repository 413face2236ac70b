"""The power-of-2 operand scales of the 3xFP16 forward, checked on the CPU.

The kernel derives pow2_floor(2^c / max(x, 1e-30)) -- the largest power of 2 not above the
correctly rounded float32 quotient, clamped to [2^-126, 2^127] -- from the exponent and
mantissa bits of max(x, 1e-30) alone, without a division: for y = m 2^e (m in [1, 2)) the
quotient is 2^(c-e) when m = 1 and lies strictly between 2^(c-e-1) and 2^(c-e) otherwise,
and a correctly rounded float32 quotient of such a y never rounds up to 2^(c-e). This test
restates both forms in numpy float32 and checks they agree on every input class the weights
and the (possibly overflowed) jet bounds can produce (the kernel uses c = 4 for the weight
scale and c = 14 for the operand scales), infinity included.
"""

from __future__ import annotations

import numpy as np
import pytest


def pow2_floor(x: np.ndarray) -> np.ndarray:
    """Largest power of 2 <= x, x clamped to [2^-126, 1.7e38] (the kernel's first form)."""
    x = np.minimum(np.maximum(x, np.float32(1.17549435e-38)), np.float32(1.7e38))
    bits = x.astype(np.float32).view(np.uint32) & np.uint32(0x7F800000)
    return bits.view(np.float32)


def by_division(c: int, x: np.ndarray) -> np.ndarray:
    y = np.fmax(x.astype(np.float32), np.float32(1e-30))  # fmaxf: the non-NaN operand wins
    with np.errstate(divide="ignore", over="ignore"):
        return pow2_floor(np.float32(2.0**c) / y)


def by_exponent(c: int, x: np.ndarray) -> np.ndarray:
    b = np.fmax(x.astype(np.float32), np.float32(1e-30)).view(np.uint32).astype(np.int64)
    k = c - ((b >> 23) - 127) - ((b & 0x7FFFFF) != 0).astype(np.int64)
    k = np.where(b >= 0x7F800000, -126, k)  # an infinite bound divides to 0
    k = np.clip(k, -126, 127)
    return ((k + 127) << 23).astype(np.uint32).view(np.float32)


def _inputs() -> np.ndarray:
    rng = np.random.default_rng(0)
    random_bits = rng.integers(0, 0x7F800000, size=2_000_000, dtype=np.uint32).view(np.float32)
    powers = np.float32(2.0) ** np.arange(-149, 128, dtype=np.float64).astype(np.float32)
    near = np.concatenate([np.nextafter(powers, np.float32(0)), np.nextafter(powers, np.float32(np.inf))])
    special = np.array([0.0, -0.0, 1e-30, 1e-31, 1.17549435e-38, 1.4e-45, 1.7e38, 3.4e38,
                        np.inf, np.nan, -1.0, 16.0, 16384.0], dtype=np.float32)
    return np.concatenate([random_bits, powers, near, special]).astype(np.float32)


@pytest.mark.parametrize("c", [4, 14])
def test_exponent_form_equals_the_divided_floor(c: int) -> None:
    x = _inputs()
    expect, got = by_division(c, x), by_exponent(c, x)
    bad = np.nonzero(expect.view(np.uint32) != got.view(np.uint32))[0]
    assert bad.size == 0, [(float(x[i]), float(expect[i]), float(got[i])) for i in bad[:5]]


def test_scales_are_powers_of_two_in_range() -> None:
    got = by_exponent(14, _inputs())
    bits = got.view(np.uint32)
    assert np.all((bits & 0x7FFFFF) == 0)  # no mantissa bits: exact powers of 2
    assert np.all(got >= np.float32(2.0**-126)) and np.all(got <= np.float32(2.0**127))


def _tf32_bits(x: np.ndarray) -> np.ndarray:
    """The kernels' TF32 rounding (tcgen05.cuh: to_tf32) on the float32 bit pattern."""
    b = x.astype(np.float32).view(np.uint32)
    return ((b.astype(np.uint64) + 0x1000) & 0xFFFFE000).astype(np.uint32)


def _tf32_nearest_ties_away(x: np.ndarray) -> np.ndarray:
    """Round float32 values to 10 explicit mantissa bits, nearest with ties away from zero,
    in float64 arithmetic (exact for these magnitudes): the definition of cvt.rna.tf32."""
    x = x.astype(np.float64)
    out = np.zeros_like(x)
    nz = (x != 0) & np.isfinite(x)
    a = np.abs(x[nz])
    e = np.floor(np.log2(a))
    e = np.where(2.0**e > a, e - 1, e)           # guard log2 rounding at powers of two
    e = np.where(2.0 ** (e + 1) <= a, e + 1, e)
    ulp = 2.0 ** (np.maximum(e, -126) - 10)     # subnormals keep the 2^-136 step
    out[nz] = np.sign(x[nz]) * np.floor(a / ulp + 0.5) * ulp
    keep = ~np.isfinite(x) | (x == 0)  # infinities, and zeros with their sign
    out[keep] = x[keep]
    return out.astype(np.float32).view(np.uint32)


def test_tf32_bit_rounding_is_nearest_ties_away() -> None:
    rng = np.random.default_rng(3)
    bits = rng.integers(0, 2**32, size=400_000, dtype=np.uint64).astype(np.uint32)
    x = bits.view(np.float32)
    x = x[np.isfinite(x)]
    # exact ties and their neighbours, around 1 and in the subnormal range
    base = np.array([1.0, 1.5, -3.25, 1e-40, -7e-39, 65504.0, 3.0e38], np.float32)
    tie = (base.view(np.uint32) | 0x1000).view(np.float32)
    extra = np.concatenate([base, tie, np.nextafter(tie, np.float32(0)),
                            np.nextafter(tie, np.float32(np.inf)),
                            np.array([np.inf, -np.inf, 0.0, -0.0], np.float32)])
    for v in (x, extra):
        got = _tf32_bits(v)
        want = _tf32_nearest_ties_away(v)
        finite = np.isfinite(v)
        np.testing.assert_array_equal(got[finite], want[finite])
    # infinities stay infinite; the largest finite values round up to infinity
    assert _tf32_bits(np.array([np.inf], np.float32))[0] == 0x7F800000
    assert _tf32_bits(np.array([np.float32(3.4028235e38)]))[0] == 0x7F800000
