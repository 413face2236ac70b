"""Host-side logic on the CPU: parameter ABI, registry, sharding, binding validation."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import fused_hoad
from fused_hoad import (
    BACKENDS,
    DEFAULT_POISSON_MLP,
    POISSON_PARAMETER_COUNT,
    POISSON_PARAMETER_LAYOUT,
    bind_model_to_flat,
    build_mlp,
    pack_poisson_parameters,
    shard_range,
    unpack_poisson_parameters,
)
from fused_hoad._extension import BUILD_HINT
from oracle import jet


def test_layout_offsets_match_the_abi_header() -> None:
    # csrc/mlp_abi.cuh:8-17: kLayer0Bias=128, kHiddenBase=192, kHiddenStride=4160,
    # kOutputBase=12672, kParameterCount=12737
    assert POISSON_PARAMETER_COUNT == 12737
    assert POISSON_PARAMETER_LAYOUT[0].bias_offset == 128
    assert POISSON_PARAMETER_LAYOUT[1].weight_offset == 192
    assert POISSON_PARAMETER_LAYOUT[2].weight_offset - POISSON_PARAMETER_LAYOUT[1].weight_offset == 4160
    assert POISSON_PARAMETER_LAYOUT[4].weight_offset == 12672
    assert [(s.weight_offset, s.bias_offset) for s in POISSON_PARAMETER_LAYOUT] == [
        (w, b) for w, b, _, _ in jet.layer_offsets()
    ]


def test_pack_of_seed0_model_matches_reference_golden(golden) -> None:
    torch.manual_seed(0)
    model = build_mlp(DEFAULT_POISSON_MLP)
    np.testing.assert_array_equal(pack_poisson_parameters(model).numpy(), golden["params_seed0"])


def test_differentiable_pack_and_unpack_round_trip() -> None:
    torch.manual_seed(3)
    model = build_mlp()
    flat = pack_poisson_parameters(model, differentiable=True)
    assert flat.requires_grad
    flat.sum().backward()
    assert all(torch.all(p.grad == 1) for p in model.parameters())
    views = unpack_poisson_parameters(flat.detach())
    for layer, spec in zip(
        [m for m in model if isinstance(m, torch.nn.Linear)], POISSON_PARAMETER_LAYOUT
    ):
        assert torch.equal(views[f"{spec.name}.weight"], layer.weight.detach())
        assert torch.equal(views[f"{spec.name}.bias"], layer.bias.detach())
    with pytest.raises(ValueError):
        unpack_poisson_parameters(torch.zeros(5))


def test_pack_rejects_wrong_shapes() -> None:
    with pytest.raises(ValueError, match="linear layers"):
        pack_poisson_parameters(torch.nn.Sequential(torch.nn.Linear(2, 64)))
    bad = build_mlp()
    bad[0] = torch.nn.Linear(3, 64)
    with pytest.raises(ValueError, match="layer0.weight"):
        pack_poisson_parameters(bad)


def test_bind_model_to_flat_makes_views() -> None:
    torch.manual_seed(0)
    model = build_mlp()
    reference = model(torch.ones(3, 2)).detach()
    flat = pack_poisson_parameters(model).clone()
    bind_model_to_flat(model, flat)
    torch.testing.assert_close(model(torch.ones(3, 2)).detach(), reference)
    flat.zero_()
    assert torch.all(model[0].weight == 0)


def test_registry_has_the_reference_fused_names() -> None:
    for name in ("fused_cuda_v0", "fused_cuda_v1", "fused_cuda", "fused_cuda_tf32",
                 "fused_cuda_tf32_pipelined", "fused_cuda_tf32_16warp", "fused_cuda_bwd_v1",
                 "fused_cuda_bwd_v2", "fused_cuda_bwd_v3", "fused_cuda_bwd_v4",
                 "fused_cuda_bwd_v5"):
        assert name in BACKENDS
    with pytest.raises(KeyError, match="fused_cuda"):
        fused_hoad.get_backend("does-not-exist")
    with pytest.raises(ValueError, match="backward"):
        fused_hoad.fused_laplacian(build_mlp(), torch.zeros(2, 2), backward="recompute")


@pytest.mark.parametrize("total", [0, 1, 7, 64, 1000, 65536, 16_777_216])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_range_partitions_contiguously(total: int, world: int) -> None:
    ranges = [shard_range(total, r, world) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == total
    for (a, b), (c, _) in zip(ranges, ranges[1:]):
        assert b == c
    sizes = [b - a for a, b in ranges]
    assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(total, world, world)


def test_binding_validates_like_the_reference() -> None:
    # csrc/bindings.cpp:9-24 messages; the device checks run before any kernel
    params = torch.zeros(POISSON_PARAMETER_COUNT)
    with pytest.raises(RuntimeError, match="CUDA"):
        fused_hoad.fused_forward_laplacian(torch.zeros(4, 2), params)
    with pytest.raises(RuntimeError, match="version"):
        fused_hoad.fused_forward_laplacian(torch.zeros(4, 2), params, 7)
    with pytest.raises(RuntimeError, match="version"):
        fused_hoad.load_extension().fused_forward_laplacian_backward(
            torch.zeros(4, 2), params, torch.zeros(4), torch.zeros(4), 0
        )


def test_missing_extension_message_is_actionable() -> None:
    assert "build.py" in BUILD_HINT and "sm_100" in BUILD_HINT


def test_trainer_rejects_cpu_parameters() -> None:
    with pytest.raises(ValueError, match="CUDA"):
        fused_hoad.PoissonTrainer(torch.zeros(POISSON_PARAMETER_COUNT))


def test_pack_cache_tracks_model_identity_and_in_place_updates() -> None:
    """The reference's pack-cache contract (tests/test_backends.py:137-148): cached per
    model, re-packed after an in-place update, and never another model's buffer."""
    from fused_hoad.backends.fused import _packed_parameters

    with torch.no_grad():
        first = build_mlp(DEFAULT_POISSON_MLP)
        packed = _packed_parameters(first)
        assert _packed_parameters(first) is packed
        first[0].weight.mul_(2.0)
        torch.testing.assert_close(_packed_parameters(first), pack_poisson_parameters(first))
        second = build_mlp(DEFAULT_POISSON_MLP)
        torch.testing.assert_close(_packed_parameters(second), pack_poisson_parameters(second))
        torch.testing.assert_close(_packed_parameters(first), pack_poisson_parameters(first))


def test_pack_cache_hands_out_a_bound_flat_buffer_without_copying() -> None:
    from fused_hoad.backends.fused import _packed_parameters

    torch.manual_seed(4)
    model = build_mlp()
    flat = pack_poisson_parameters(model).clone()
    bind_model_to_flat(model, flat)
    with torch.no_grad():
        packed = _packed_parameters(model)
        assert packed.data_ptr() == flat.data_ptr() and torch.equal(packed, flat)
        flat.mul_(0.5)  # an update of the buffer is the model's update
        assert torch.equal(_packed_parameters(model), flat)
    # while autograd records, the pack is differentiable and reaches the module parameters
    differentiable = _packed_parameters(model)
    assert differentiable.requires_grad
    differentiable.sum().backward()
    assert all(torch.all(p.grad == 1) for p in model.parameters())


def test_layout_table_is_contiguous_and_ordered() -> None:
    offset = 0
    for spec in POISSON_PARAMETER_LAYOUT:
        assert spec.weight_offset == offset
        assert spec.bias_offset == offset + spec.out_features * spec.in_features
        assert spec.weight_elements == spec.out_features * spec.in_features
        offset = spec.end_offset
    assert offset == POISSON_PARAMETER_COUNT
