"""Ordering of the training step's dependent launches.

The step kernel starts while the weight pre-split still runs, and the update kernel starts
while the step kernel still runs; each reads some inputs before it waits on the device for
the kernel before it (the step kernel its points and parameters, the update kernel the
parameters and Adam moments). These tests change that state with ordinary torch kernels in
the same stream right before each step, vary the batch between steps (so the grid size, and
with it the number of SMs the update kernel can take early, changes), and require the fused
step to give bitwise what the separate launches give (gradient kernel, then Adam) on the
same state — eagerly and as CUDA-graph replays.
"""

from __future__ import annotations

import pytest
import torch
from helpers import PARAMETER_COUNT, read_status

import fused_hoad
from fused_hoad import uniform_points
from oracle import jet

pytestmark = pytest.mark.gpu

HYPER = (1e-3, 0.9, 0.999, 1e-8)  # lr, beta1, beta2, eps


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    read_status()
    yield


def _state(params: torch.Tensor):
    return [params.clone(), torch.zeros_like(params), torch.zeros_like(params),
            torch.zeros(1, dtype=torch.int64, device=params.device)]


def _disturb(state, k: int) -> None:
    """Rewrite the parameters and both moments in place (ordinary torch kernels)."""
    p, m, v, _ = state
    p.mul_(1.0 + 0.01 * (k + 1))
    m.mul_(0.5).add_(1e-4)
    v.add_(1e-7 * (k + 1))


def _separate_step(C, state, x, xb, kernel: int) -> torch.Tensor:
    p, m, v, s = state
    want = C.pinn_step_gradients(x, xb, p, len(x), len(xb), 100.0, kernel)
    C.adam_step(p, want[:PARAMETER_COUNT], m, v, s, *HYPER)
    return want


@pytest.mark.parametrize("kernel", [6, 5])
def test_step_sees_state_written_right_before_it(kernel: int) -> None:
    C = fused_hoad.load_extension()
    params = jet.init_parameters(3).cuda()
    xb = jet.boundary_points(256, seed=9).cuda()
    fused, separate = _state(params), _state(params)
    ex = C.exchange_create(1, 0, 5.0, 0)
    try:
        # 100 interior + 256 boundary points are 3 tiles (a grid of 4 CTAs with the
        # tensor-core kernel: the update kernel's CTAs take the other SMs while the step
        # kernel runs); 65,536 fills every SM for several tiles.
        for k, n in enumerate((65_536, 100, 20_000, 100, 65_536)):
            x = uniform_points(n, seed=40 + k).cuda()
            _disturb(fused, k)
            _disturb(separate, k)
            grad = torch.empty(PARAMETER_COUNT + 1, device="cuda")
            loss = C.train_step(x, xb, *fused, *HYPER, len(x), len(xb), 100.0, ex, kernel,
                                grad)
            want = _separate_step(C, separate, x, xb, kernel)
            assert torch.equal(grad, want), k
            assert torch.equal(loss, want[PARAMETER_COUNT:]), k
            for got, ref in zip(fused, separate):
                assert torch.equal(got, ref), k
    finally:
        C.exchange_destroy(ex)
    assert read_status() == 0


def test_graph_replays_see_state_written_between_them() -> None:
    C = fused_hoad.load_extension()
    params = jet.init_parameters(4).cuda()
    x = uniform_points(30_000, seed=50).cuda()
    xb = jet.boundary_points(128, seed=10).cuda()
    fused, separate = _state(params), _state(params)
    grad = torch.empty(PARAMETER_COUNT + 1, device="cuda")
    ex = C.exchange_create(1, 0, 5.0, 0)
    try:
        # one eager step first: sets the kernels' attributes and advances both the same way
        C.train_step(x, xb, *fused, *HYPER, len(x), len(xb), 100.0, ex, 6, grad)
        _separate_step(C, separate, x, xb, 6)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            C.train_step(x, xb, *fused, *HYPER, len(x), len(xb), 100.0, ex, 6, grad)
        # capture launched nothing: the state is the one after the eager step
        for k in range(3):
            _disturb(fused, k)
            _disturb(separate, k)
            graph.replay()
            want = _separate_step(C, separate, x, xb, 6)
            assert torch.equal(grad, want), k
            for got, ref in zip(fused, separate):
                assert torch.equal(got, ref), k
        torch.cuda.synchronize()
        del graph
    finally:
        C.exchange_destroy(ex)
    assert read_status() == 0
