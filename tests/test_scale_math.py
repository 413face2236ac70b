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
