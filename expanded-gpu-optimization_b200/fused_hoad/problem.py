"""The fixed Poisson MLP contract and the manufactured Poisson problem.

Only what callers of the fused path need: the shape contract ``MLPConfig`` /
``DEFAULT_POISSON_MLP`` and ``build_mlp`` (reference ``src/fused_hoad/specs.py:9-22``,
``models.py:15-26``, ``problems/poisson.py:15-21``), and the manufactured solution and
source ``f = -2 pi^2 sin(pi x) sin(pi y)`` (``problems/poisson.py:29-39``) that the
training loss uses.
"""

from __future__ import annotations

from dataclasses import dataclass
from math import pi

import torch
from torch import Tensor, nn


# Hidden activations with a fused jet (reference src/fused_hoad/models.py:9-12): tanh, the
# reference kernels' activation, and SiLU, the other jet of its forward-Laplacian backend.
ACTIVATIONS: dict[str, type[nn.Module]] = {"tanh": nn.Tanh, "silu": nn.SiLU}


@dataclass(frozen=True, slots=True)
class MLPConfig:
    """Shape contract of the MLP targeted by the fused kernels."""

    input_dim: int
    hidden_dim: int
    hidden_layers: int
    output_dim: int = 1
    activation: str = "tanh"

    def __post_init__(self) -> None:
        for name in ("input_dim", "hidden_dim", "hidden_layers", "output_dim"):
            if getattr(self, name) < 1:
                raise ValueError(f"{name} must be positive")
        if self.activation not in ACTIVATIONS:
            raise ValueError(f"activation must be one of {tuple(ACTIVATIONS)}")


DEFAULT_POISSON_MLP = MLPConfig(input_dim=2, hidden_dim=64, hidden_layers=4)


def build_mlp(config: MLPConfig = DEFAULT_POISSON_MLP) -> nn.Sequential:
    """``Linear, activation`` x hidden_layers then ``Linear``, with nn.Linear's default init
    (reference ``src/fused_hoad/models.py:15-26``)."""
    layers: list[nn.Module] = []
    width = config.input_dim
    for _ in range(config.hidden_layers):
        layers += [nn.Linear(width, config.hidden_dim), ACTIVATIONS[config.activation]()]
        width = config.hidden_dim
    layers.append(nn.Linear(width, config.output_dim))
    return nn.Sequential(*layers)


def _check(coordinates: Tensor) -> None:
    if coordinates.ndim != 2 or coordinates.shape[1] != 2:
        raise ValueError("Poisson coordinates must have shape [batch, 2]")


def manufactured_solution(coordinates: Tensor) -> Tensor:
    """``sin(pi x) sin(pi y)`` on ``[-1, 1]^2``, shape ``[batch, 1]``."""
    _check(coordinates)
    return torch.sin(pi * coordinates[:, 0:1]) * torch.sin(pi * coordinates[:, 1:2])


def manufactured_source(coordinates: Tensor) -> Tensor:
    """``f = Laplacian(u*) = -2 pi^2 sin(pi x) sin(pi y)``, shape ``[batch, 1]``."""
    return -2.0 * pi**2 * manufactured_solution(coordinates)


def uniform_points(
    count: int, *, seed: int = 1, device: str | torch.device = "cpu"
) -> Tensor:
    """Collocation points uniform in ``[-1, 1]^2``: drawn on a CPU generator, then moved.

    CPU and CUDA generators give different streams; drawing on the CPU keeps the points
    identical on every device (the benchmark configs use seed 1).
    """
    generator = torch.Generator().manual_seed(seed)
    points = torch.rand(count, 2, generator=generator) * 2 - 1
    return points.to(device)
