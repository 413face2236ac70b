"""ctypes front end for the FP64 C restatement ``oracle/c/jet64.c`` (test only)."""

from __future__ import annotations

import ctypes
from functools import lru_cache

import numpy as np

from oracle.build import build_c_oracle

PARAMETER_COUNT = 12737
_dp = ctypes.POINTER(ctypes.c_double)


@lru_cache(maxsize=1)
def _lib() -> ctypes.CDLL:
    lib = ctypes.CDLL(str(build_c_oracle()))
    lib.jet64_forward.argtypes = [_dp, _dp, ctypes.c_int64, _dp, _dp]
    lib.jet64_backward.argtypes = [_dp, _dp, _dp, _dp, ctypes.c_int64, _dp, _dp]
    lib.jet64_parameter_count.restype = ctypes.c_int
    assert lib.jet64_parameter_count() == PARAMETER_COUNT
    return lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(_dp)


def _f64(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float64))


def forward(params, coords) -> tuple[np.ndarray, np.ndarray]:
    """(u [n], lap [n]) in FP64."""
    p, x = _f64(params), _f64(coords).reshape(-1, 2)
    n = x.shape[0]
    u, lap = np.empty(n), np.empty(n)
    _lib().jet64_forward(_ptr(p), _ptr(x), n, _ptr(u), _ptr(lap))
    return u, lap


def backward(params, coords, grad_u, grad_lap) -> tuple[np.ndarray, np.ndarray]:
    """(grad_params [12737], grad_coords [n, 2]) in FP64 via the closed-form adjoint."""
    p, x = _f64(params), _f64(coords).reshape(-1, 2)
    gu, gl = _f64(grad_u).reshape(-1), _f64(grad_lap).reshape(-1)
    n = x.shape[0]
    gp, gx = np.empty(PARAMETER_COUNT), np.empty((n, 2))
    _lib().jet64_backward(_ptr(p), _ptr(x), _ptr(gu), _ptr(gl), n, _ptr(gp), _ptr(gx))
    return gp, gx
