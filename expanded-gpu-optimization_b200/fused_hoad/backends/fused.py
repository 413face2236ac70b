"""Fused CUDA backend: ``model -> (u, Laplacian u)`` in one sm_100a kernel launch.

The reference's public surface (``src/fused_hoad/backends/fused.py``): the autograd function
``FusedForwardLaplacian``, the pack cache ``_packed_parameters`` and
``fused_laplacian(model, x, version=2, backward="cuda")`` with its backward-mode names. The
backward is always one of the fused adjoint kernels; the reference's PyTorch "recompute"
backward is an oracle and lives in the test suite's ``oracle`` package, not here.
"""

from __future__ import annotations

import weakref

import torch
from torch import Tensor, nn

from fused_hoad._extension import fused_forward_laplacian, fused_forward_laplacian_backward
from fused_hoad.parameters import flat_buffer_of, pack_poisson_parameters
from fused_hoad.problem import ACTIVATIONS

# Backward-mode names callers pass (the reference's), and the backward kernel version each
# selects: "cuda" is version 6 (tensor cores), "cuda_vN" is version N (FP32 CUDA cores).
_CUDA_BACKWARD_VERSIONS = {"cuda": 6, **{f"cuda_v{k}": k for k in range(1, 6)}}
BACKWARD_MODES = tuple(_CUDA_BACKWARD_VERSIONS)


class FusedForwardLaplacian(torch.autograd.Function):
    """``(u, lap)`` from the fused forward kernel; gradients for the coordinates and the
    flat parameters from one fused backward kernel. Autograd hands the backward zero tensors
    for an output that received no gradient (materialised gradients, the default)."""

    @staticmethod
    def forward(ctx, coordinates: Tensor, parameters: Tensor, version: int, backward: str,
                activation: str = "tanh"):
        ctx.kernel = (_CUDA_BACKWARD_VERSIONS[backward], activation)
        ctx.save_for_backward(coordinates, parameters)
        return fused_forward_laplacian(coordinates, parameters, version, activation)

    @staticmethod
    def backward(ctx, grad_output: Tensor, grad_laplacian: Tensor):
        coordinates, parameters = ctx.saved_tensors
        want_x, want_p = ctx.needs_input_grad[:2]
        if not (want_x or want_p):
            return None, None, None, None, None
        bwd_version, activation = ctx.kernel
        grad_p, grad_x = fused_forward_laplacian_backward(
            coordinates, parameters, grad_output, grad_laplacian, bwd_version, activation
        )
        return (grad_x if want_x else None), (grad_p if want_p else None), None, None, None


class _PackEntry:
    """What the pack cache holds for one model."""

    __slots__ = ("tensors", "versions", "packed")

    def __init__(self, tensors: list[Tensor]) -> None:
        self.tensors = tensors
        self.versions: tuple[int, ...] | None = None
        self.packed: Tensor | None = None


# One entry per live model, dropped with the model (no id() reuse hazard).
_pack_cache: "weakref.WeakKeyDictionary[nn.Module, _PackEntry]" = weakref.WeakKeyDictionary()


def _packed_parameters(model: nn.Module) -> Tensor:
    """The model's flat ABI buffer for a kernel call.

    While autograd records (grad enabled and a parameter requires grad) this is a fresh
    differentiable pack, so gradients reach the model's parameters. Otherwise it is reused
    until a parameter's version counter moves (an in-place update such as an optimizer step)
    and re-packed then; a model whose parameters are already views of one flat buffer
    (``bind_model_to_flat``) hands out that buffer itself and never copies.
    """
    entry = _pack_cache.get(model)
    if entry is None:
        entry = _PackEntry(list(model.parameters()))
        _pack_cache[model] = entry
    if torch.is_grad_enabled() and any(t.requires_grad for t in entry.tensors):
        return pack_poisson_parameters(model, differentiable=True)
    versions = tuple(t._version for t in entry.tensors)
    if entry.packed is None or versions != entry.versions:
        bound = flat_buffer_of(model)
        entry.packed = bound if bound is not None else pack_poisson_parameters(model)
        entry.versions = versions
    return entry.packed


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
    ``"cuda_vN"``; all run a fused adjoint kernel). The hidden activation (tanh or SiLU)
    is read from the model.
    """
    if backward not in BACKWARD_MODES:
        raise ValueError(f"backward must be one of {BACKWARD_MODES}")
    activation = model_activation(model)
    parameters = _packed_parameters(model)
    coordinates = coordinates.contiguous()
    if parameters.requires_grad or coordinates.requires_grad:
        return FusedForwardLaplacian.apply(coordinates, parameters, version, backward, activation)
    return fused_forward_laplacian(coordinates, parameters, version, activation)
