"""Fused CUDA backend: ``model -> (u, Laplacian u)`` in one sm_100a kernel launch.

Mirrors the reference's ``src/fused_hoad/backends/fused.py:1-138``: the autograd function
``FusedForwardLaplacian``, the weakref-keyed pack cache ``_packed_parameters`` and
``fused_laplacian(model, x, version=2, backward="cuda")``. The backward is always the fused
adjoint-jet kernel; the reference's PyTorch "recompute" backward is an oracle and lives in
the test suite's ``oracle`` package, not here.
"""

from __future__ import annotations

import weakref

import torch
from torch import Tensor, nn

from fused_hoad._extension import fused_forward_laplacian, fused_forward_laplacian_backward
from fused_hoad.parameters import pack_poisson_parameters
from fused_hoad.problem import ACTIVATIONS

_cache: dict[str, object] = {}

# Backward modes kept for drop-in compatibility with the reference's names
# (backends/fused.py:24-32); every one runs the single fused adjoint kernel.
_CUDA_BACKWARD_VERSIONS = {
    "cuda": 6,
    "cuda_v1": 1,
    "cuda_v2": 2,
    "cuda_v3": 3,
    "cuda_v4": 4,
    "cuda_v5": 5,
}
BACKWARD_MODES = tuple(_CUDA_BACKWARD_VERSIONS)


class FusedForwardLaplacian(torch.autograd.Function):
    """Fused-kernel forward ``(u, lap)``; fused-kernel backward to ``(coords, params)``."""

    @staticmethod
    def forward(
        ctx,
        coordinates: Tensor,
        parameters: Tensor,
        version: int,
        backward: str,
        activation: str = "tanh",
    ):
        ctx.save_for_backward(coordinates, parameters)
        ctx.backward_mode = backward
        ctx.activation = activation
        return fused_forward_laplacian(coordinates, parameters, version, activation)

    @staticmethod
    def backward(ctx, grad_output: Tensor | None, grad_laplacian: Tensor | None):
        coordinates, parameters = ctx.saved_tensors
        needs_coordinates, needs_parameters = ctx.needs_input_grad[:2]
        if grad_output is None:
            grad_output = torch.zeros_like(coordinates[:, :1])
        if grad_laplacian is None:
            grad_laplacian = torch.zeros_like(coordinates[:, :1])
        grad_parameters, grad_coordinates = fused_forward_laplacian_backward(
            coordinates,
            parameters,
            grad_output,
            grad_laplacian,
            _CUDA_BACKWARD_VERSIONS[ctx.backward_mode],
            ctx.activation,
        )
        return (
            grad_coordinates if needs_coordinates else None,
            grad_parameters if needs_parameters else None,
            None,
            None,
            None,
        )


def _packed_parameters(model: nn.Module) -> Tensor:
    """Differentiable pack when training; otherwise pack once per in-place weight update.

    The parameter list is cached per model through a weakref, and the packed buffer is
    rebuilt only when a parameter's version counter moved (reference fused.py:104-121).
    """
    model_ref = _cache.get("model")
    if model_ref is None or model_ref() is not model:
        _cache.clear()
        _cache.update(model=weakref.ref(model), parameters=list(model.parameters()))
    parameters = _cache["parameters"]
    if torch.is_grad_enabled() and any(p.requires_grad for p in parameters):
        return pack_poisson_parameters(model, differentiable=True)
    versions = [p._version for p in parameters]
    if versions != _cache.get("versions"):
        _cache.update(versions=versions, packed=pack_poisson_parameters(model))
    return _cache["packed"]


def model_activation(model: nn.Module) -> str:
    """Name of the model's hidden activation (``"tanh"`` or ``"silu"``), all layers alike."""
    kinds = {name for module in model.modules() for name, cls in ACTIVATIONS.items()
             if type(module) is cls}
    if len(kinds) != 1:
        raise TypeError(f"the fused kernels need one hidden activation out of {tuple(ACTIVATIONS)}")
    return kinds.pop()


def fused_laplacian(
    model: nn.Module, coordinates: Tensor, version: int = 2, backward: str = "cuda"
) -> tuple[Tensor, Tensor]:
    """Evaluate the fixed Poisson MLP and its input Laplacian with one CUDA kernel.

    ``backward`` names the gradient path when autograd is active (``"cuda"`` or
    ``"cuda_vN"``; all run the fused adjoint kernel). The hidden activation (tanh or SiLU)
    is read from the model.
    """
    if backward not in BACKWARD_MODES:
        raise ValueError(f"backward must be one of {BACKWARD_MODES}")
    activation = model_activation(model)
    parameters = _packed_parameters(model)
    if parameters.requires_grad or coordinates.requires_grad:
        return FusedForwardLaplacian.apply(
            coordinates.contiguous(), parameters, version, backward, activation
        )
    return fused_forward_laplacian(coordinates.contiguous(), parameters, version, activation)
