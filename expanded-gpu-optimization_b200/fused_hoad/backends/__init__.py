"""Registry of the fused backends under the reference's names.

The reference registers ``fused_cuda*`` backends in ``BACKENDS`` only when its extension
is built (``src/fused_hoad/backends/__init__.py:37-67``). This package holds only the
fused hot path, so the registry holds only those names, each mapped onto the sm_100a
kernels: forward versions 0-2 are the FP32 CUDA-core kernel, 3 the 3xFP16 tensor-core
kernel and 4-5 the 3xTF32 one; ``fused_cuda`` and every ``bwd`` name use the fused adjoint
kernels (backward 6, the default, on the tensor cores; 1-5 on the FP32 CUDA cores). The
reference's PyTorch backends (eager, forward_laplacian, func, compiled) are not part of this
package.
"""

from __future__ import annotations

from collections.abc import Callable
from functools import partial

from torch import Tensor, nn

from fused_hoad.backends.fused import fused_laplacian

Backend = Callable[[nn.Module, Tensor], tuple[Tensor, Tensor]]

BACKENDS: dict[str, Backend] = {
    "fused_cuda_v0": partial(fused_laplacian, version=0),
    "fused_cuda_v1": partial(fused_laplacian, version=1),
    "fused_cuda": fused_laplacian,
    "fused_cuda_tf32": partial(fused_laplacian, version=3),
    "fused_cuda_tf32_pipelined": partial(fused_laplacian, version=4),
    "fused_cuda_tf32_16warp": partial(fused_laplacian, version=5),
    "fused_cuda_bwd_v1": partial(fused_laplacian, backward="cuda_v1"),
    "fused_cuda_bwd_v2": partial(fused_laplacian, backward="cuda_v2"),
    "fused_cuda_bwd_v3": partial(fused_laplacian, backward="cuda_v3"),
    "fused_cuda_bwd_v4": partial(fused_laplacian, backward="cuda_v4"),
    "fused_cuda_bwd_v5": partial(fused_laplacian, backward="cuda_v5"),
}
FIXED_CONTRACT_BACKENDS: tuple[str, ...] = tuple(BACKENDS)


def get_backend(name: str) -> Backend:
    """Return the backend registered under ``name``."""
    try:
        return BACKENDS[name]
    except KeyError:
        available = ", ".join(sorted(BACKENDS))
        raise KeyError(f"unknown backend {name!r}; available: {available}") from None


__all__ = ["BACKENDS", "FIXED_CONTRACT_BACKENDS", "Backend", "fused_laplacian", "get_backend"]
