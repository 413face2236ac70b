"""Shared helpers for the parity tests: C-ABI calls through ctypes, oracle comparisons."""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from fused_hoad import _native

PARAMETER_COUNT = 12737


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle() -> int:
    return torch.cuda.current_stream().cuda_stream


def capi_forward(coords: torch.Tensor, params: torch.Tensor, version: int):
    """u, lap through ``fhb_forward`` (C ABI)."""
    lib = _native.library()
    n = coords.shape[0]
    u = torch.empty(n, 1, device=coords.device)
    lap = torch.empty(n, 1, device=coords.device)
    code = lib.fhb_forward(
        ptr(coords), ptr(params), ptr(u), ptr(lap), n, version, stream_handle()
    )
    _native.check(code, "fhb_forward")
    return u, lap


def capi_backward(coords, params, grad_u, grad_lap, version: int = 6):
    """(grad_params, grad_coords) through ``fhb_backward`` (C ABI)."""
    lib = _native.library()
    n = coords.shape[0]
    grad_p = torch.empty(PARAMETER_COUNT, device=coords.device)
    grad_x = torch.empty(n, 2, device=coords.device)
    ws_bytes = lib.fhb_backward_workspace_bytes(n)
    workspace = torch.empty(max(1, (ws_bytes + 3) // 4), device=coords.device)
    code = lib.fhb_backward(
        ptr(coords), ptr(params), ptr(grad_u), ptr(grad_lap), ptr(grad_p), ptr(grad_x), n,
        version, ptr(workspace), ws_bytes, stream_handle(),
    )
    _native.check(code, "fhb_backward")
    return grad_p, grad_x


def read_status(device: int = 0) -> int:
    lib = _native.library()
    out = ctypes.c_uint(0)
    _native.check(lib.fhb_read_device_status(device, ctypes.byref(out)), "read status")
    return int(out.value)


def scaled_error(actual, expected) -> tuple[float, float]:
    a = np.asarray(actual.detach().cpu() if torch.is_tensor(actual) else actual, np.float64)
    e = np.asarray(expected.detach().cpu() if torch.is_tensor(expected) else expected, np.float64)
    return float(np.abs(a - e).max()), float(np.abs(e).max())


def assert_scaled(actual, expected, tolerance: float, what: str = "") -> None:
    """max|actual - expected| <= tolerance * max|expected| (reference tests/test_fused.py:180-184)."""
    error, scale = scaled_error(actual, expected)
    assert error <= tolerance * scale, f"{what}: max error {error:.3e} vs scale {scale:.3e}"
