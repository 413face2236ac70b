"""Shared pytest setup: the ``gpu`` marker, import paths and the golden fixtures."""

from __future__ import annotations

import sys
from functools import lru_cache
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
PACKAGE_DIR = ROOT / "expanded-gpu-optimization_b200"
for entry in (str(ROOT), str(PACKAGE_DIR)):
    if entry not in sys.path:
        sys.path.insert(0, entry)

GOLDEN = Path(__file__).resolve().parent / "golden" / "golden.npz"


def pytest_configure(config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@lru_cache(maxsize=1)
def _golden() -> dict[str, np.ndarray]:
    with np.load(GOLDEN) as data:
        return {key: data[key] for key in data.files}


@pytest.fixture(scope="session")
def golden() -> dict[str, np.ndarray]:
    return _golden()


def assert_scaled_close(actual, expected, tolerance: float, what: str = "") -> None:
    """max|actual - expected| <= tolerance * max|expected| (tests/test_fused.py:180-184)."""
    actual = np.asarray(actual, dtype=np.float64)
    expected = np.asarray(expected, dtype=np.float64)
    assert actual.shape == expected.shape, (what, actual.shape, expected.shape)
    scale = float(np.abs(expected).max()) if expected.size else 0.0
    error = float(np.abs(actual - expected).max()) if expected.size else 0.0
    assert error <= tolerance * scale, f"{what}: max error {error:.3e} vs scale {scale:.3e}"
