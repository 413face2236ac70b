"""SiLU hidden activation on the GPU: the forward kernels (FP32 versions 0-2, tensor-core
versions 3-5 in 3xTF32 form), the FP32 adjoint kernel (every backward version), the fused
autograd backend and the trainer, against the oracle and the reference's golden vectors.

SiLU is the other jet of the reference's PyTorch forward-Laplacian backend
(src/fused_hoad/backends/forward_laplacian.py:34-38); the reference's fused CUDA path is
tanh only, so the golden gradients come from autograd through its forward Laplacian.
Tolerances are the tanh tests': forward atol 1e-5 / rtol 1e-4 (tests/test_fused.py:34-35),
saturated weights and gradients <= 1e-4 of the largest magnitude (:48-49, :180-218).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from helpers import PARAMETER_COUNT, assert_scaled, ptr, stream_handle

import fused_hoad
from fused_hoad import MLPConfig, _native, build_mlp, uniform_points
from fused_hoad.parameters import pack_poisson_parameters
from oracle import jet

pytestmark = pytest.mark.gpu

FORWARD_VERSIONS = [0, 1, 2, 3, 4, 5]
BACKWARD_VERSIONS = [1, 5, 6]
SILU = 1  # FHB_ACTIVATION_SILU


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    yield


def _params(seed: int = 0, scale: float = 1.0) -> torch.Tensor:
    return jet.init_parameters(seed, scale).cuda()


@pytest.mark.parametrize("version", FORWARD_VERSIONS)
@pytest.mark.parametrize("batch", [1, 33, 129, 1_000, 65_536])
def test_silu_forward_matches_oracle(batch: int, version: int) -> None:
    params = _params()
    x = uniform_points(batch, seed=61)
    u, lap = fused_hoad.fused_forward_laplacian(x.cuda(), params, version, "silu")
    eu, el = jet.forward_laplacian(params.cpu(), x, "silu")
    torch.testing.assert_close(u.cpu(), eu, atol=1e-5, rtol=1e-4)
    torch.testing.assert_close(lap.cpu(), el, atol=1e-5, rtol=1e-4)


@pytest.mark.parametrize("version", FORWARD_VERSIONS)
def test_silu_forward_matches_reference_golden(golden, version: int) -> None:
    params = torch.from_numpy(golden["silu_params_seed0"]).cuda()
    for n in (1, 33, 129, 1000):
        x = torch.from_numpy(golden[f"silufwd{n}_x"]).cuda()
        u, lap = fused_hoad.fused_forward_laplacian(x, params, version, "silu")
        np.testing.assert_allclose(u.cpu().numpy(), golden[f"silufwd{n}_u64"], atol=1e-5,
                                   rtol=1e-4)
        np.testing.assert_allclose(lap.cpu().numpy(), golden[f"silufwd{n}_lap64"], atol=1e-5,
                                   rtol=1e-4)


@pytest.mark.parametrize("version", FORWARD_VERSIONS)
def test_silu_forward_saturated_weights_against_fp64(golden, version: int) -> None:
    params = torch.from_numpy(golden["silu_params_seed1_x3"]).cuda()
    x = torch.from_numpy(golden["silusat_x"]).cuda()
    u, lap = fused_hoad.fused_forward_laplacian(x, params, version, "silu")
    assert_scaled(u.cpu(), golden["silusat_u64"], 1e-4, "u")
    assert_scaled(lap.cpu(), golden["silusat_lap64"], 1e-4, "lap")


def test_silu_tensor_core_versions_agree_and_differ_from_tanh() -> None:
    """Versions 3-5 run one kernel for SiLU (3xTF32), so they agree bitwise; the activation
    really switches (SiLU and tanh results differ)."""
    params = _params()
    x = uniform_points(10_000, seed=62).cuda()
    outs = [fused_hoad.fused_forward_laplacian(x, params, v, "silu") for v in (3, 4, 5)]
    for u, lap in outs[1:]:
        assert torch.equal(u, outs[0][0]) and torch.equal(lap, outs[0][1])
    tu, _ = fused_hoad.fused_forward_laplacian(x, params, 4, "tanh")
    assert not torch.allclose(tu, outs[0][0])


@pytest.mark.parametrize("version", BACKWARD_VERSIONS)
@pytest.mark.parametrize("batch", [1, 33, 1_000, 20_000])
def test_silu_backward_matches_oracle(batch: int, version: int) -> None:
    params = _params()
    x = uniform_points(batch, seed=63)
    g = torch.Generator().manual_seed(3)
    gu, gl = torch.randn(batch, generator=g), torch.randn(batch, generator=g)
    gp, gx = fused_hoad.fused_forward_laplacian_backward(
        x.cuda(), params, gu.cuda(), gl.cuda(), version, "silu"
    )
    ep, ex = jet.recompute_backward(params.cpu().double(), x.double(), gu.double(),
                                    gl.double(), "silu")
    assert_scaled(gp.cpu(), ep, 1e-4, "grad params")
    assert_scaled(gx.cpu(), ex, 1e-4, "grad coords")


@pytest.mark.parametrize("version", BACKWARD_VERSIONS)
def test_silu_backward_against_reference_golden(golden, version: int) -> None:
    params = torch.from_numpy(golden["silu_params_seed0"]).cuda()
    for n in (33, 1000):
        gp, gx = fused_hoad.fused_forward_laplacian_backward(
            torch.from_numpy(golden[f"silubwd{n}_x"]).cuda(), params,
            torch.from_numpy(golden[f"silubwd{n}_gu"]).cuda(),
            torch.from_numpy(golden[f"silubwd{n}_gl"]).cuda(), version, "silu",
        )
        # per parameter block, as the reference's tests (tests/test_fused.py:180-218)
        want = golden[f"silubwd{n}_gp64"]
        for start, stop in ((0, 128), (128, 192), (192, 4288), (4288, 4352),
                            (12608, 12672), (12672, 12737)):
            assert_scaled(gp.cpu()[start:stop], want[start:stop], 1e-4, f"block {start}")
        assert_scaled(gx.cpu(), golden[f"silubwd{n}_gx64"], 1e-4, "grad coords")


def test_silu_backward_versions_use_one_kernel_and_reproduce() -> None:
    params = _params()
    x = uniform_points(5_000, seed=64).cuda()
    gu, gl = torch.randn(5_000, device="cuda"), torch.randn(5_000, device="cuda")
    first = fused_hoad.fused_forward_laplacian_backward(x, params, gu, gl, 6, "silu")
    for version in (1, 5, 6):
        again = fused_hoad.fused_forward_laplacian_backward(x, params, gu, gl, version, "silu")
        assert torch.equal(first[0], again[0]) and torch.equal(first[1], again[1])


def test_silu_capi_matches_torch_binding_and_rejects_unknown_activation() -> None:
    lib = _native.library()
    params = _params()
    x = uniform_points(3_000, seed=65).cuda()
    u = torch.empty(3_000, 1, device="cuda")
    lap = torch.empty(3_000, 1, device="cuda")
    _native.check(lib.fhb_forward_ex(ptr(x), ptr(params), ptr(u), ptr(lap), 3_000, 4, SILU,
                                     stream_handle()), "fhb_forward_ex")
    bu, bl = fused_hoad.fused_forward_laplacian(x, params, 4, "silu")
    assert torch.equal(u, bu) and torch.equal(lap, bl)
    assert lib.fhb_forward_ex(ptr(x), ptr(params), ptr(u), ptr(lap), 3_000, 4, 7,
                              stream_handle()) == 1
    gp = torch.empty(PARAMETER_COUNT, device="cuda")
    gx = torch.empty(3_000, 2, device="cuda")
    gu, gl = torch.randn(3_000, device="cuda"), torch.randn(3_000, device="cuda")
    ws_bytes = lib.fhb_backward_workspace_bytes(3_000)
    ws = torch.empty((ws_bytes + 15) // 16 * 4, device="cuda")
    _native.check(lib.fhb_backward_ex(ptr(x), ptr(params), ptr(gu), ptr(gl), ptr(gp), ptr(gx),
                                      3_000, 6, SILU, ptr(ws), ws_bytes, stream_handle()),
                  "fhb_backward_ex")
    bp, bx = fused_hoad.fused_forward_laplacian_backward(x, params, gu, gl, 6, "silu")
    assert torch.equal(gp, bp) and torch.equal(gx, bx)
    with pytest.raises(RuntimeError, match="activation"):
        fused_hoad.fused_forward_laplacian(x, params, 2, "relu")


def test_silu_model_trains_through_the_fused_backend_like_the_reference(golden) -> None:
    """torch.optim.Adam on a SiLU model through fused_laplacian (forward kernel + FP32
    adjoint kernel) follows the reference's 5-step FL trajectory."""
    torch.manual_seed(0)
    model = build_mlp(MLPConfig(2, 64, 4, activation="silu")).cuda()
    np.testing.assert_array_equal(pack_poisson_parameters(model).detach().cpu().numpy(),
                                  golden["silu_params_seed0"])
    x = torch.from_numpy(golden["adam_x"]).cuda()
    f = fused_hoad.manufactured_source(x)
    optimizer = torch.optim.Adam(model.parameters(), lr=1e-3, betas=(0.9, 0.999))
    losses = []
    for _ in range(len(golden["siluadam_losses"])):
        optimizer.zero_grad()
        _, lap = fused_hoad.fused_laplacian(model, x, version=2)
        loss = (lap - f).pow(2).mean()
        loss.backward()
        optimizer.step()
        losses.append(loss.item())
    np.testing.assert_allclose(losses, golden["siluadam_losses"], rtol=1e-4)
    diff = np.abs(pack_poisson_parameters(model).detach().cpu().numpy()
                  - golden["siluadam_params_final"])
    assert np.mean(diff > 1e-5) < 1e-3, float(diff.max())


@pytest.mark.parametrize("exchange", ["peer", "nccl"])
def test_silu_trainer_follows_the_reference_trajectory(golden, exchange: str) -> None:
    torch.manual_seed(0)
    model = build_mlp(MLPConfig(2, 64, 4, activation="silu")).cuda()
    trainer = fused_hoad.PoissonTrainer(model, exchange=exchange)
    assert trainer.activation == "silu"
    x = torch.from_numpy(golden["adam_x"]).cuda()
    losses = [trainer.step(x).item() for _ in range(len(golden["siluadam_losses"]))]
    np.testing.assert_allclose(losses, golden["siluadam_losses"], rtol=1e-4)
    diff = np.abs(trainer.params.cpu().numpy() - golden["siluadam_params_final"])
    assert np.mean(diff > 1e-5) < 1e-3, float(diff.max())
    trainer.close()


def test_silu_trainer_with_boundary_follows_the_oracle() -> None:
    params = _params()
    x = uniform_points(2_048, seed=66)
    xb = jet.boundary_points(256, seed=6)
    trainer = fused_hoad.PoissonTrainer(params.clone(), activation="silu")
    losses = [trainer.step(x.cuda(), boundary=xb.cuda()).item() for _ in range(4)]
    p = params.cpu().clone()
    m, v = torch.zeros_like(p), torch.zeros_like(p)
    want = []
    for step in range(1, 5):
        loss, grad = jet.pinn_step_gradients(p, x, xb, activation="silu")
        want.append(loss.item())
        jet.adam_update(p, grad, m, v, step)
    np.testing.assert_allclose(losses, want, rtol=1e-4)
    diff = (trainer.params.cpu() - p).abs()
    assert float((diff > 1e-5).float().mean()) < 1e-3, float(diff.max())
    with pytest.raises(ValueError, match="does not match"):
        fused_hoad.PoissonTrainer(build_mlp().cuda(), activation="silu")
    trainer.close()
