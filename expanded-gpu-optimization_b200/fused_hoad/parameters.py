"""The flat-parameter ABI of the fixed Poisson MLP (12,737 floats).

The buffer the kernels read (``include/fused_hoad_b200.h``, the reference's
``csrc/mlp_abi.cuh:8-17`` and ``src/fused_hoad/parameters.py``): the linear layers of the
width chain 2 -> 64 -> 64 -> 64 -> 64 -> 1 one after another, each as its ``weight``
``[out, in]`` (row-major, ``nn.Linear`` order) followed by its ``bias`` ``[out]``. The public
names (``POISSON_PARAMETER_LAYOUT``, ``POISSON_PARAMETER_COUNT``, ``ParameterSlice``,
``pack_poisson_parameters``, ``unpack_poisson_parameters``) are the reference's.
"""

from __future__ import annotations

from itertools import accumulate
from typing import NamedTuple

import torch
from torch import Tensor, nn

# Widths of the MLP's layers: input, four hidden layers, output.
WIDTHS = (2, 64, 64, 64, 64, 1)


class ParameterSlice(NamedTuple):
    """Where one linear layer lives in the flat buffer."""

    name: str
    out_features: int
    in_features: int
    weight_offset: int
    bias_offset: int
    weight_elements: int
    end_offset: int


def _abi_table(widths: tuple[int, ...]) -> tuple[ParameterSlice, ...]:
    """One entry per consecutive width pair; a layer's block is its weight, then its bias."""
    pairs = list(zip(widths[1:], widths[:-1]))  # (out, in)
    blocks = [o * i + o for o, i in pairs]
    starts = [0, *accumulate(blocks)][:-1]
    return tuple(
        ParameterSlice(f"layer{k}", o, i, start, start + o * i, o * i, start + block)
        for k, ((o, i), start, block) in enumerate(zip(pairs, starts, blocks))
    )


POISSON_PARAMETER_LAYOUT = _abi_table(WIDTHS)
POISSON_PARAMETER_COUNT = POISSON_PARAMETER_LAYOUT[-1].end_offset
assert POISSON_PARAMETER_COUNT == 12737
# Sizes of the buffer's pieces in order: weight, bias, weight, bias, ...
_PIECE_SIZES = [n for s in POISSON_PARAMETER_LAYOUT for n in (s.weight_elements, s.out_features)]


def linear_layers(model: nn.Module) -> list[nn.Linear]:
    """The model's ``nn.Linear`` modules in registration order."""
    return [module for module in model.modules() if isinstance(module, nn.Linear)]


def _abi_tensors(model: nn.Module) -> list[Tensor]:
    """The model's weights and biases in buffer order, after checking every shape against
    the ABI (ValueError naming the first layer that does not fit)."""
    layers = linear_layers(model)
    if len(layers) != len(POISSON_PARAMETER_LAYOUT):
        raise ValueError(
            f"expected {len(POISSON_PARAMETER_LAYOUT)} linear layers, found {len(layers)}"
        )
    want = [((s.out_features, s.in_features), (s.out_features,))
            for s in POISSON_PARAMETER_LAYOUT]
    have = [(tuple(m.weight.shape), None if m.bias is None else tuple(m.bias.shape))
            for m in layers]
    if have != want:
        k = next(k for k, (h, w) in enumerate(zip(have, want)) if h != w)
        name = POISSON_PARAMETER_LAYOUT[k].name
        if have[k][0] != want[k][0]:
            raise ValueError(f"{name}.weight must have shape {want[k][0]}, got {have[k][0]}")
        raise ValueError(f"{name}.bias must have shape {want[k][1]}, got {have[k][1]}")
    return [t for m in layers for t in (m.weight, m.bias)]


def _views(flat: Tensor) -> list[Tensor]:
    """Shaped views (weight, bias, weight, ...) into a flat buffer."""
    pieces = torch.split(flat, _PIECE_SIZES)
    views: list[Tensor] = []
    for spec, weight, bias in zip(POISSON_PARAMETER_LAYOUT, pieces[0::2], pieces[1::2]):
        views += [weight.view(spec.out_features, spec.in_features), bias]
    return views


def pack_poisson_parameters(model: nn.Module, *, differentiable: bool = False) -> Tensor:
    """The model's parameters as one contiguous ABI buffer.

    ``differentiable=True``: a concatenation that autograd tracks, so a gradient on the
    buffer reaches the model (the reference's ``torch.cat`` pack). Otherwise a detached copy:
    one multi-tensor copy into a buffer allocated on the parameters' device and dtype.
    """
    tensors = _abi_tensors(model)
    if differentiable:
        return nn.utils.parameters_to_vector(tensors)
    flat = torch.empty(POISSON_PARAMETER_COUNT, dtype=tensors[0].dtype,
                       device=tensors[0].device)
    with torch.no_grad():
        torch._foreach_copy_(_views(flat), [t.detach() for t in tensors])
    return flat


def unpack_poisson_parameters(parameters: Tensor) -> dict[str, Tensor]:
    """Views ``{"layerK.weight": [out, in], "layerK.bias": [out]}`` into a packed buffer."""
    if parameters.ndim != 1 or parameters.numel() != POISSON_PARAMETER_COUNT:
        raise ValueError(f"parameters must have shape [{POISSON_PARAMETER_COUNT}]")
    names = [f"{s.name}.{kind}" for s in POISSON_PARAMETER_LAYOUT
             for kind in ("weight", "bias")]
    return dict(zip(names, _views(parameters)))


def bind_model_to_flat(model: nn.Module, flat: Tensor) -> None:
    """Make every parameter of ``model`` a view into ``flat`` (same ABI order).

    After this, an in-place update of ``flat`` (the fused Adam kernel) is the model's
    update and no per-step pack is needed. ``flat`` must already hold the packed values.
    """
    for tensor, view in zip(_abi_tensors(model), _views(flat)):
        tensor.data = view


def flat_buffer_of(model: nn.Module) -> Tensor | None:
    """The flat ABI buffer the model's parameters are views of (``bind_model_to_flat``), or
    None when they are separate tensors."""
    tensors = _abi_tensors(model)
    first = tensors[0]
    if first.storage_offset() != 0:
        return None
    storage = first.untyped_storage()
    offset = 0
    for tensor, size in zip(tensors, _PIECE_SIZES):
        if (tensor.untyped_storage().data_ptr() != storage.data_ptr()
                or tensor.storage_offset() != offset or not tensor.is_contiguous()):
            return None
        offset += size
    if storage.nbytes() < POISSON_PARAMETER_COUNT * first.element_size():
        return None
    flat = first.new_empty(0).set_(storage, 0, (POISSON_PARAMETER_COUNT,), (1,))
    return flat.detach()
