"""ctypes view of the C ABI (``include/fused_hoad_b200.h``) in ``libfused_hoad_b200.so``.

This is how a non-torch host (or a test) drives the kernels: raw device pointers, sizes
and a ``cudaStream_t`` as an integer. Signatures here must match the header.
"""

from __future__ import annotations

import ctypes
from functools import lru_cache
from pathlib import Path

LIBRARY = Path(__file__).resolve().parent / "libfused_hoad_b200.so"
HEADER = Path(__file__).resolve().parents[2] / "include" / "fused_hoad_b200.h"

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_SIGNATURES: dict[str, tuple[object, list]] = {
    "fhb_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "fhb_last_cuda_error": (ctypes.c_int, []),
    "fhb_parameter_count": (ctypes.c_int, []),
    "fhb_prepare_device": (ctypes.c_int, [ctypes.c_int]),
    "fhb_forward": (ctypes.c_int, [_p, _p, _p, _p, _i64, ctypes.c_int, _p]),
    "fhb_forward_ex": (ctypes.c_int, [_p, _p, _p, _p, _i64, ctypes.c_int, ctypes.c_int, _p]),
    "fhb_forward_biharmonic": (ctypes.c_int, [_p, _p, _p, _p, _p, _i64, _p]),
    "fhb_backward_workspace_bytes": (ctypes.c_size_t, [_i64]),
    "fhb_backward": (
        ctypes.c_int,
        [_p, _p, _p, _p, _p, _p, _i64, ctypes.c_int, _p, ctypes.c_size_t, _p],
    ),
    "fhb_backward_ex": (
        ctypes.c_int,
        [_p, _p, _p, _p, _p, _p, _i64, ctypes.c_int, ctypes.c_int, _p, ctypes.c_size_t, _p],
    ),
    "fhb_backward_noalloc": (ctypes.c_int, [_p, _p, _p, _p, _p, _p, _i64, _p]),
    "fhb_poisson_step_gradients": (
        ctypes.c_int,
        [_p, _p, _i64, _i64, _p, _p, _p, _p, ctypes.c_int, _p, ctypes.c_size_t, _p],
    ),
    "fhb_pinn_step_workspace_bytes": (ctypes.c_size_t, [_i64, _i64]),
    "fhb_pinn_step_gradients": (
        ctypes.c_int,
        [_p, _i64, _i64, _p, _i64, _i64, ctypes.c_float, _p, _p, _p, ctypes.c_int,
         ctypes.c_int, _p, ctypes.c_size_t, _p],
    ),
    "fhb_adam_step": (
        ctypes.c_int,
        [_p, _p, _p, _p, _i64, _p, ctypes.c_float, ctypes.c_float, ctypes.c_float,
         ctypes.c_float, _p],
    ),
    "fhb_exchange_buffer_bytes": (ctypes.c_size_t, []),
    "fhb_exchange_create": (
        ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_uint64, ctypes.POINTER(_p)]
    ),
    "fhb_exchange_handle": (ctypes.c_int, [_p, _p]),
    "fhb_exchange_connect": (ctypes.c_int, [_p, _p]),
    "fhb_exchange_buffer": (ctypes.c_int, [_p, ctypes.POINTER(_p)]),
    "fhb_debug_exchange_connect_local": (ctypes.c_int, [_p, ctypes.POINTER(_p)]),
    "fhb_exchange_destroy": (ctypes.c_int, [_p]),
    "fhb_train_step": (
        ctypes.c_int,
        [_p, _i64, _i64, _p, _i64, _i64, ctypes.c_float, _p, _p, _p, _p, ctypes.c_float,
         ctypes.c_float, ctypes.c_float, ctypes.c_float, _p, _p, _p, ctypes.c_int,
         ctypes.c_int, _p, ctypes.c_size_t, _p],
    ),
    "fhb_read_device_status": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_uint)]),
    "fhb_debug_bounded_wait_selftest": (ctypes.c_int, [ctypes.c_uint64, _p]),
    "fhb_debug_tanh": (ctypes.c_int, [_p, _p, _i64, ctypes.c_int, _p]),
}


@lru_cache(maxsize=1)
def library() -> ctypes.CDLL:
    """Load the C-ABI library (torch is imported first so libcudart is resolvable)."""
    import torch  # noqa: F401  (loads the CUDA runtime the library links against)

    if not LIBRARY.exists():
        raise RuntimeError(
            f"{LIBRARY.name} is not built; run `python expanded-gpu-optimization_b200/build.py`"
        )
    lib = ctypes.CDLL(str(LIBRARY))
    for name, (restype, argtypes) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


def status_string(code: int) -> str:
    return library().fhb_status_string(code).decode()


def check(code: int, what: str) -> None:
    if code != 0:
        raise RuntimeError(f"{what} failed: {status_string(code)} (code {code})")
