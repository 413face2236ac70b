"""The flat-parameter ABI of the fixed Poisson MLP (12,737 floats).

Same layout and same public names as the reference's ``src/fused_hoad/parameters.py:1-100``
(and ``csrc/mlp_abi.cuh:8-17``): per linear layer, ``weight`` [out, in] row-major then
``bias`` [out], for the layers 2->64, 64->64 (x3), 64->1.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor, nn


@dataclass(frozen=True, slots=True)
class ParameterSlice:
    """Offsets and shape of one linear layer in the flat parameter buffer."""

    name: str
    out_features: int
    in_features: int
    weight_offset: int
    bias_offset: int

    @property
    def weight_elements(self) -> int:
        return self.out_features * self.in_features

    @property
    def end_offset(self) -> int:
        return self.bias_offset + self.out_features


LAYER_SHAPES = ((64, 2), (64, 64), (64, 64), (64, 64), (1, 64))


def _layout() -> tuple[ParameterSlice, ...]:
    slices, offset = [], 0
    for index, (out_features, in_features) in enumerate(LAYER_SHAPES):
        weight_elements = out_features * in_features
        slices.append(
            ParameterSlice(
                f"layer{index}", out_features, in_features, offset, offset + weight_elements
            )
        )
        offset += weight_elements + out_features
    return tuple(slices)


POISSON_PARAMETER_LAYOUT = _layout()
POISSON_PARAMETER_COUNT = POISSON_PARAMETER_LAYOUT[-1].end_offset
assert POISSON_PARAMETER_COUNT == 12737


def linear_layers(model: nn.Module) -> list[nn.Linear]:
    return [module for module in model.modules() if isinstance(module, nn.Linear)]


def _segments(model: nn.Module) -> list[Tensor]:
    layers = linear_layers(model)
    if len(layers) != len(POISSON_PARAMETER_LAYOUT):
        raise ValueError(f"expected {len(POISSON_PARAMETER_LAYOUT)} linear layers")
    segments: list[Tensor] = []
    for layer, spec in zip(layers, POISSON_PARAMETER_LAYOUT, strict=True):
        expected = (spec.out_features, spec.in_features)
        if tuple(layer.weight.shape) != expected:
            raise ValueError(
                f"{spec.name}.weight must have shape {expected}, got {tuple(layer.weight.shape)}"
            )
        if layer.bias is None or tuple(layer.bias.shape) != (spec.out_features,):
            raise ValueError(f"{spec.name}.bias must have shape ({spec.out_features},)")
        segments.extend((layer.weight.reshape(-1), layer.bias.reshape(-1)))
    return segments


def pack_poisson_parameters(model: nn.Module, *, differentiable: bool = False) -> Tensor:
    """Pack the 2x64x64x64x64x1 MLP into the flat ABI buffer.

    ``differentiable=True`` returns a ``torch.cat`` so gradients flow back to the model
    (reference ``parameters.py:77-78``); otherwise a detached contiguous copy.
    """
    segments = _segments(model)
    if differentiable:
        return torch.cat(segments)
    packed = segments[0].new_empty(POISSON_PARAMETER_COUNT)
    offset = 0
    for segment in segments:
        packed[offset : offset + segment.numel()].copy_(segment.detach())
        offset += segment.numel()
    return packed


def unpack_poisson_parameters(parameters: Tensor) -> dict[str, Tensor]:
    """Shaped views ``{"layerK.weight", "layerK.bias"}`` into a packed buffer."""
    if parameters.ndim != 1 or parameters.numel() != POISSON_PARAMETER_COUNT:
        raise ValueError(f"parameters must have shape [{POISSON_PARAMETER_COUNT}]")
    views: dict[str, Tensor] = {}
    for spec in POISSON_PARAMETER_LAYOUT:
        end = spec.weight_offset + spec.weight_elements
        views[f"{spec.name}.weight"] = parameters[spec.weight_offset : end].view(
            spec.out_features, spec.in_features
        )
        views[f"{spec.name}.bias"] = parameters[spec.bias_offset : spec.end_offset]
    return views


def bind_model_to_flat(model: nn.Module, flat: Tensor) -> None:
    """Make every parameter of ``model`` a view into ``flat`` (same ABI order).

    After this, an in-place update of ``flat`` (the fused Adam kernel) is the model's
    update and no per-step pack is needed. ``flat`` must already hold the packed values.
    """
    views = unpack_poisson_parameters(flat)
    for layer, spec in zip(linear_layers(model), POISSON_PARAMETER_LAYOUT, strict=True):
        layer.weight.data = views[f"{spec.name}.weight"]
        layer.bias.data = views[f"{spec.name}.bias"]
