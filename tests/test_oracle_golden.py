"""Pin both CPU oracles to the golden vectors recorded from the unmodified reference."""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import assert_scaled_close

from oracle import cjet, jet

FORWARD_BATCHES = (1, 2, 15, 16, 17, 31, 32, 33, 63, 64, 65, 127, 128, 129, 1000, 1024)


def test_parameter_init_matches_reference_pack(golden) -> None:
    # build_mlp + pack_poisson_parameters (src/fused_hoad/parameters.py:55-84)
    np.testing.assert_array_equal(jet.init_parameters(0).numpy(), golden["params_seed0"])
    np.testing.assert_array_equal(
        jet.init_parameters(1, scale=3.0).numpy(), golden["params_seed1_x3"]
    )


def test_points_match_reference_generator(golden) -> None:
    for n in FORWARD_BATCHES:
        np.testing.assert_array_equal(jet.uniform_points(n).numpy(), golden[f"fwd{n}_x"])


@pytest.mark.parametrize("n", FORWARD_BATCHES)
def test_torch_oracle_forward_fp32_matches_reference(golden, n: int) -> None:
    params = torch.from_numpy(golden["params_seed0"])
    x = torch.from_numpy(golden[f"fwd{n}_x"])
    u, lap = jet.forward_laplacian(params, x)
    # Same ops in the same order as the reference: agreement to FP32 rounding.
    np.testing.assert_allclose(u.numpy(), golden[f"fwd{n}_u32"], rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(lap.numpy(), golden[f"fwd{n}_lap32"], rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("n", FORWARD_BATCHES)
def test_torch_oracle_forward_fp64_matches_reference(golden, n: int) -> None:
    params = torch.from_numpy(golden["params_seed0"]).double()
    x = torch.from_numpy(golden[f"fwd{n}_x"]).double()
    u, lap = jet.forward_laplacian(params, x)
    np.testing.assert_allclose(u.numpy(), golden[f"fwd{n}_u64"], rtol=1e-12, atol=1e-14)
    np.testing.assert_allclose(lap.numpy(), golden[f"fwd{n}_lap64"], rtol=1e-12, atol=1e-14)


@pytest.mark.parametrize("n", (1, 33, 1000))
def test_torch_oracle_eager_matches_reference(golden, n: int) -> None:
    params = torch.from_numpy(golden["params_seed0"]).double()
    x = torch.from_numpy(golden[f"fwd{n}_x"]).double()
    _, lap = jet.eager_laplacian(params, x)
    np.testing.assert_allclose(lap.numpy(), golden[f"fwd{n}_eager_lap64"], rtol=1e-10, atol=1e-12)


@pytest.mark.parametrize("n", FORWARD_BATCHES)
def test_c_oracle_forward_matches_reference_fp64(golden, n: int) -> None:
    u, lap = cjet.forward(golden["params_seed0"], golden[f"fwd{n}_x"])
    np.testing.assert_allclose(u, golden[f"fwd{n}_u64"][:, 0], rtol=1e-11, atol=1e-13)
    np.testing.assert_allclose(lap, golden[f"fwd{n}_lap64"][:, 0], rtol=1e-11, atol=1e-13)


def test_oracles_match_reference_on_saturated_weights(golden) -> None:
    params = golden["params_seed1_x3"]
    u, lap = cjet.forward(params, golden["sat_x"])
    assert_scaled_close(lap, golden["sat_lap64"][:, 0], 1e-12, "c lap")
    assert_scaled_close(u, golden["sat_u64"][:, 0], 1e-12, "c u")
    tu, tl = jet.forward_laplacian(torch.from_numpy(params), torch.from_numpy(golden["sat_x"]))
    np.testing.assert_allclose(tl.numpy(), golden["sat_lap32"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("n", (1, 15, 16, 17, 33, 1000))
def test_torch_oracle_backward_fp32_matches_reference(golden, n: int) -> None:
    params = torch.from_numpy(golden["params_seed0"])
    gp, gx = jet.recompute_backward(
        params,
        torch.from_numpy(golden[f"bwd{n}_x"]),
        torch.from_numpy(golden[f"bwd{n}_gu"]),
        torch.from_numpy(golden[f"bwd{n}_gl"]),
    )
    assert_scaled_close(gp.numpy(), golden[f"bwd{n}_gp32"], 1e-6, "grad params")
    assert_scaled_close(gx.numpy(), golden[f"bwd{n}_gx32"], 1e-6, "grad coords")


@pytest.mark.parametrize("n", (33, 1000))
def test_c_oracle_backward_matches_reference_fp64(golden, n: int) -> None:
    gp, gx = cjet.backward(
        golden["params_seed0"], golden[f"bwd{n}_x"], golden[f"bwd{n}_gu"], golden[f"bwd{n}_gl"]
    )
    assert_scaled_close(gp, golden[f"bwd{n}_gp64"], 1e-11, "grad params")
    assert_scaled_close(gx, golden[f"bwd{n}_gx64"], 1e-11, "grad coords")
    # every parameter block, not just the max (tests/test_fused.py:209-218)
    for w, b, o, i in jet.layer_offsets():
        assert_scaled_close(gp[w : w + o * i], golden[f"bwd{n}_gp64"][w : w + o * i], 1e-11)
        assert_scaled_close(gp[b : b + o], golden[f"bwd{n}_gp64"][b : b + o], 1e-11)


def test_c_oracle_backward_matches_reference_saturated(golden) -> None:
    gp, gx = cjet.backward(
        golden["params_seed1_x3"], golden["satbwd_x"], golden["satbwd_gu"], golden["satbwd_gl"]
    )
    assert_scaled_close(gp, golden["satbwd_gp64"], 1e-11, "grad params")
    assert_scaled_close(gx, golden["satbwd_gx64"], 1e-11, "grad coords")


def test_oracle_adam_trajectory_matches_reference(golden) -> None:
    params = torch.from_numpy(golden["params_seed0"]).clone()
    x = torch.from_numpy(golden["adam_x"])
    m, v = torch.zeros_like(params), torch.zeros_like(params)
    losses = []
    for step in range(1, len(golden["adam_losses"]) + 1):
        loss, grad, _ = jet.poisson_step_gradients(params, x)
        losses.append(loss.item())
        jet.adam_update(params, grad, m, v, step)
    np.testing.assert_allclose(losses, golden["adam_losses"], rtol=1e-5)
    np.testing.assert_allclose(params.numpy(), golden["adam_params_final"], rtol=1e-5, atol=1e-7)


def test_oracle_pinn_loss_matches_reference(golden) -> None:
    """Interior residual + 100 * mean(u^2) on the boundary (reference training.py:68-94)."""
    params = torch.from_numpy(golden["params_seed0"])
    xb = torch.from_numpy(golden["pinn_xb"])
    np.testing.assert_array_equal(jet.boundary_points(len(xb), seed=2).numpy(), golden["pinn_xb"])
    loss, grad = jet.pinn_step_gradients(params, torch.from_numpy(golden["pinn_x"]), xb)
    np.testing.assert_allclose(loss.item(), float(golden["pinn_loss"]), rtol=1e-5)
    assert_scaled_close(grad, golden["pinn_grad"], 1e-5, "PINN grad params")


def test_known_answers() -> None:
    # With every weight and bias zero except b_out the network is constant, so u = b_out
    # and lap = 0 exactly (the analogue of tests/test_backends.py:104-108's linear case).
    params = torch.zeros(jet.PARAMETER_COUNT, dtype=torch.float64)
    params[-1] = 0.25
    x = jet.uniform_points(17, dtype=torch.float64)
    u, lap = jet.forward_laplacian(params, x)
    assert torch.all(u == 0.25) and torch.all(lap == 0.0)
    cu, cl = cjet.forward(params.numpy(), x.numpy())
    assert np.all(cu == 0.25) and np.all(cl == 0.0)


# ---------------------------------------------------------------- SiLU (f rank 4) ----

SILU_FORWARD_BATCHES = (1, 33, 129, 1000)


def test_silu_parameters_match_reference_pack(golden) -> None:
    # nn.Linear init does not depend on the activation module, so the SiLU MLP of seed 0
    # packs to the tanh MLP's buffer
    np.testing.assert_array_equal(golden["silu_params_seed0"], golden["params_seed0"])


@pytest.mark.parametrize("n", SILU_FORWARD_BATCHES)
def test_torch_oracle_silu_forward_matches_reference(golden, n: int) -> None:
    params = torch.from_numpy(golden["silu_params_seed0"])
    x = torch.from_numpy(golden[f"silufwd{n}_x"])
    u, lap = jet.forward_laplacian(params, x, "silu")
    np.testing.assert_allclose(u.numpy(), golden[f"silufwd{n}_u32"], rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(lap.numpy(), golden[f"silufwd{n}_lap32"], rtol=1e-6, atol=1e-7)
    u, lap = jet.forward_laplacian(params.double(), x.double(), "silu")
    np.testing.assert_allclose(u.numpy(), golden[f"silufwd{n}_u64"], rtol=1e-12, atol=1e-14)
    np.testing.assert_allclose(lap.numpy(), golden[f"silufwd{n}_lap64"], rtol=1e-12, atol=1e-14)
    _, lap = jet.eager_laplacian(params.double(), x.double(), "silu")
    np.testing.assert_allclose(lap.numpy(), golden[f"silufwd{n}_eager_lap64"], rtol=1e-10,
                               atol=1e-12)


def test_torch_oracle_silu_saturated_forward_matches_reference(golden) -> None:
    params = torch.from_numpy(golden["silu_params_seed1_x3"]).double()
    u, lap = jet.forward_laplacian(params, torch.from_numpy(golden["silusat_x"]).double(), "silu")
    assert_scaled_close(u.numpy(), golden["silusat_u64"], 1e-12, "u")
    assert_scaled_close(lap.numpy(), golden["silusat_lap64"], 1e-12, "lap")


@pytest.mark.parametrize("n", (33, 1000))
def test_torch_oracle_silu_backward_matches_reference(golden, n: int) -> None:
    params = torch.from_numpy(golden["silu_params_seed0"]).double()
    gp, gx = jet.recompute_backward(
        params,
        torch.from_numpy(golden[f"silubwd{n}_x"]).double(),
        torch.from_numpy(golden[f"silubwd{n}_gu"]).double(),
        torch.from_numpy(golden[f"silubwd{n}_gl"]).double(),
        "silu",
    )
    assert_scaled_close(gp.numpy(), golden[f"silubwd{n}_gp64"], 1e-11, "grad params")
    assert_scaled_close(gx.numpy(), golden[f"silubwd{n}_gx64"], 1e-11, "grad coords")


def test_oracle_silu_adam_trajectory_matches_reference(golden) -> None:
    p = torch.from_numpy(golden["silu_params_seed0"]).clone()
    x = torch.from_numpy(golden["adam_x"])
    m, v = torch.zeros_like(p), torch.zeros_like(p)
    losses = []
    for step in range(1, len(golden["siluadam_losses"]) + 1):
        loss, grad, _ = jet.poisson_step_gradients(p, x, activation="silu")
        losses.append(loss.item())
        jet.adam_update(p, grad, m, v, step)
    np.testing.assert_allclose(losses, golden["siluadam_losses"], rtol=1e-5)
    diff = np.abs(p.numpy() - golden["siluadam_params_final"])
    assert np.mean(diff > 1e-6) < 1e-3, float(diff.max())


BIHARMONIC_BATCHES = (1, 33, 129, 1000)


@pytest.mark.parametrize("n", BIHARMONIC_BATCHES)
def test_biharmonic_jet_fp64_matches_reference_autograd(golden, n: int) -> None:
    """The nine-component jet against the reference's laplacian(laplacian(u)) in FP64."""
    params = torch.from_numpy(golden["params_seed0"]).double()
    x = torch.from_numpy(golden[f"bih{n}_x"]).double()
    u, lap, bilap = jet.forward_biharmonic(params, x)
    np.testing.assert_allclose(u.numpy(), golden[f"bih{n}_u64"], rtol=1e-12, atol=1e-14)
    np.testing.assert_allclose(lap.numpy(), golden[f"bih{n}_lap64"], rtol=1e-11, atol=1e-13)
    np.testing.assert_allclose(bilap.numpy(), golden[f"bih{n}_bilap64"], rtol=1e-10, atol=1e-12)


@pytest.mark.parametrize("n", BIHARMONIC_BATCHES)
def test_biharmonic_jet_fp32_within_fp32_tolerance_of_reference(golden, n: int) -> None:
    params = torch.from_numpy(golden["params_seed0"])
    x = torch.from_numpy(golden[f"bih{n}_x"])
    u, lap, bilap = jet.forward_biharmonic(params, x)
    for got, key in ((u, "u"), (lap, "lap"), (bilap, "bilap")):
        np.testing.assert_allclose(got.numpy(), golden[f"bih{n}_{key}32"], rtol=1e-4, atol=1e-5)


def test_biharmonic_eager_oracle_matches_reference(golden) -> None:
    params = torch.from_numpy(golden["params_seed0"]).double()
    x = torch.from_numpy(golden["bih33_x"]).double()
    _, _, bilap = jet.eager_biharmonic(params, x)
    np.testing.assert_allclose(bilap.numpy(), golden["bih33_bilap64"], rtol=1e-10, atol=1e-12)


def test_biharmonic_jet_saturated_weights(golden) -> None:
    params = torch.from_numpy(golden["params_seed1_x3"]).double()
    x = torch.from_numpy(golden["bihsat_x"]).double()
    u, lap, bilap = jet.forward_biharmonic(params, x)
    assert_scaled_close(bilap.numpy(), golden["bihsat_bilap64"], 1e-10, "bilap x3")
    assert_scaled_close(lap.numpy(), golden["bihsat_lap64"], 1e-10, "lap x3")
