"""The biharmonic kernel (fhb_forward_biharmonic / fused_hoad.fused_forward_biharmonic).

The reference computes the biharmonic only by nested autograd: its ``autodiff.laplacian``
(src/fused_hoad/autodiff.py:39-41) applied to its own output. The golden vectors hold that,
from the unmodified reference in FP64 and FP32; the oracle's nine-component jet is pinned to
them on the CPU (tests/test_oracle_golden.py). Tolerance: the FP32 forward's (atol 1e-5,
rtol 1e-4; tests/test_fused.py:34-35 of the reference), and <= 1e-4 x max|FP64| for the x3
saturated weights (its :48-49).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import assert_scaled_close
from helpers import ptr, stream_handle

import fused_hoad
from fused_hoad import _native, uniform_points
from oracle import jet

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")


def _close(got: torch.Tensor, want, what: str) -> None:
    np.testing.assert_allclose(got.detach().cpu().double().numpy(), np.asarray(want, np.float64),
                               rtol=1e-4, atol=1e-5, err_msg=what)


@pytest.mark.parametrize("n", [1, 33, 129, 1000])
def test_biharmonic_matches_reference_autograd(golden, n: int) -> None:
    params = torch.from_numpy(golden["params_seed0"]).cuda()
    x = torch.from_numpy(golden[f"bih{n}_x"]).cuda()
    u, lap, bilap = fused_hoad.fused_forward_biharmonic(x, params)
    for got, key in ((u, "u"), (lap, "lap"), (bilap, "bilap")):
        _close(got, golden[f"bih{n}_{key}64"], f"{key} vs FP64 autograd, n={n}")
        _close(got, golden[f"bih{n}_{key}32"], f"{key} vs FP32 autograd, n={n}")


@pytest.mark.parametrize("n", [2, 15, 16, 17, 31, 32, 63, 64, 65, 127, 128, 4099, 65_536])
def test_biharmonic_matches_fp64_jet_oracle(n: int) -> None:
    params = jet.init_parameters(0)
    x = uniform_points(n, seed=7)
    eu, el, eb = jet.forward_biharmonic(params.double(), x.double())
    u, lap, bilap = fused_hoad.fused_forward_biharmonic(x.cuda(), params.cuda())
    _close(u, eu, "u")
    _close(lap, el, "lap")
    _close(bilap, eb, "bilap")


def test_biharmonic_saturated_weights(golden) -> None:
    params = torch.from_numpy(golden["params_seed1_x3"]).cuda()
    x = torch.from_numpy(golden["bihsat_x"]).cuda()
    u, lap, bilap = fused_hoad.fused_forward_biharmonic(x, params)
    assert_scaled_close(u.cpu().numpy(), golden["bihsat_u64"], 1e-4, "u x3")
    assert_scaled_close(lap.cpu().numpy(), golden["bihsat_lap64"], 1e-4, "lap x3")
    assert_scaled_close(bilap.cpu().numpy(), golden["bihsat_bilap64"], 1e-4, "bilap x3")


def test_biharmonic_laplacian_agrees_with_the_laplacian_kernels() -> None:
    params = jet.init_parameters(2).cuda()
    x = uniform_points(10_000, seed=8).cuda()
    u, lap, _ = fused_hoad.fused_forward_biharmonic(x, params)
    ru, rl = fused_hoad.fused_forward_laplacian(x, params, 2)
    torch.testing.assert_close(u, ru, atol=1e-5, rtol=1e-4)
    torch.testing.assert_close(lap, rl, atol=1e-5, rtol=1e-4)


def test_biharmonic_large_batch_is_pointwise_and_reproducible() -> None:
    """At 1M points: a shard gives bitwise the rows of the full batch, a rerun is bitwise
    equal, and a strided sample matches the FP64 oracle."""
    params = jet.init_parameters(0).cuda()
    x = uniform_points(1 << 20, seed=9).cuda()
    full = fused_hoad.fused_forward_biharmonic(x, params)
    again = fused_hoad.fused_forward_biharmonic(x, params)
    shard = fused_hoad.fused_forward_biharmonic(x[123_457:300_001].contiguous(), params)
    for a, b, c in zip(full, again, shard):
        assert torch.equal(a, b)
        assert torch.equal(a[123_457:300_001], c)
    rows = torch.arange(0, 1 << 20, 997)
    eu, el, eb = jet.forward_biharmonic(params.cpu().double(), x.cpu()[rows].double())
    _close(full[2].cpu()[rows], eb, "bilap sample")
    _close(full[1].cpu()[rows], el, "lap sample")


def test_biharmonic_through_the_c_abi_and_empty_batch() -> None:
    lib = _native.library()
    params = jet.init_parameters(0).cuda()
    x = uniform_points(777, seed=10).cuda()
    outs = [torch.full((777, 1), float("nan"), device="cuda") for _ in range(3)]
    code = lib.fhb_forward_biharmonic(ptr(x), ptr(params), *(ptr(o) for o in outs), 777,
                                      stream_handle())
    _native.check(code, "fhb_forward_biharmonic")
    want = fused_hoad.fused_forward_biharmonic(x, params)
    for got, ref in zip(outs, want):
        assert torch.equal(got, ref)
    empty = fused_hoad.fused_forward_biharmonic(torch.empty(0, 2, device="cuda"), params)
    assert all(t.shape == (0, 1) for t in empty)
    with pytest.raises(RuntimeError, match="float32"):
        fused_hoad.fused_forward_biharmonic(x.double(), params)
