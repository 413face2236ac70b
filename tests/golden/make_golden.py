"""Generate golden vectors from the UNMODIFIED reference package (run in the build container).

    python tests/golden/make_golden.py [--reference-src PATH]

Imports ``fused_hoad`` from the reference checkout's ``src/`` (default: the path in
``FUSED_HOAD_REFERENCE_SRC``) and records, on the CPU, the outputs of its own oracles:

* ``forward_laplacian`` (``src/fused_hoad/backends/forward_laplacian.py:95-104``) in FP32
  and FP64 and ``eager_laplacian`` (``src/fused_hoad/backends/eager.py:8-10``) in FP64,
  for the seed-0 Poisson MLP (``torch.manual_seed(0); build_mlp(DEFAULT_POISSON_MLP)``)
  at the batch sizes the reference's tests use (``tests/test_fused.py:28, :193``);
* the same with seed-1 weights scaled by 3 (saturated tanh, ``tests/test_fused.py:38-49``);
* ``_recompute_backward`` (``src/fused_hoad/backends/fused.py:76-101``) gradients for
  fixed upstream gradients;
* a 5-step ``torch.optim.Adam(lr=1e-3)`` trajectory of the interior Poisson loss
  ``mean((lap - f)^2)`` (``benchmarks/benchmark_training.py:39-57``);
* the full PINN loss of ``poisson_loss_fn`` (``src/fused_hoad/training.py:68-94``: interior
  residual + 100 * mean(u^2) on ``boundary_points``, ``:45-53``) through the FL backend, and
  its parameter gradients;
* the biharmonic: the reference's ``autodiff.laplacian`` (``src/fused_hoad/autodiff.py:39-41``)
  applied to its own output, on the seed-0 MLP in FP32 and FP64 and on the x3 seed-1 MLP in
  FP64 (u, Laplacian, biharmonic);
* for the SiLU MLP (``MLPConfig(activation="silu")``, ``src/fused_hoad/models.py:9-12``): FL
  forwards in FP32/FP64 and the FP64 eager Laplacian, an x3-scaled FP64 forward, FP64
  gradients by autograd through FL (the reference's fused backward is tanh-only), and the
  5-step Adam trajectory.

Inputs come from CPU generators (points: seed 1, ``rand*2-1``; upstream grads: seed 2).
The result is ``tests/golden/golden.npz``; nothing at test time reads the reference.
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent / "golden.npz"
FORWARD_BATCHES = (1, 2, 15, 16, 17, 31, 32, 33, 63, 64, 65, 127, 128, 129, 1000, 1024)
BACKWARD_BATCHES_F32 = (1, 15, 16, 17, 33, 1000)
BACKWARD_BATCHES_F64 = (33, 1000)
SATURATED_BATCH = 4096
SATURATED_BACKWARD_BATCH = 2048
ADAM_BATCH = 512
ADAM_STEPS = 5
PINN_INTERIOR = 256
PINN_BOUNDARY = 64
SILU_FORWARD_BATCHES = (1, 33, 129, 1000)
SILU_BACKWARD_BATCHES = (33, 1000)
BIHARMONIC_BATCHES = (1, 33, 129, 1000)
BIHARMONIC_SATURATED_BATCH = 1024


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument(
        "--reference-src",
        default=os.environ.get("FUSED_HOAD_REFERENCE_SRC"),
        help="the reference checkout's src/ directory (or FUSED_HOAD_REFERENCE_SRC)",
    )
    args = parser.parse_args()
    if not args.reference_src:
        parser.error("give --reference-src or set FUSED_HOAD_REFERENCE_SRC")
    sys.path.insert(0, args.reference_src)

    import torch
    from fused_hoad import (
        DEFAULT_POISSON_MLP,
        build_mlp,
        forward_laplacian,
        manufactured_source,
        pack_poisson_parameters,
    )
    from fused_hoad.backends.eager import eager_laplacian
    from fused_hoad.backends.fused import _recompute_backward

    torch.set_num_threads(min(8, os.cpu_count() or 1))

    def model(seed: int, scale: float = 1.0):
        torch.manual_seed(seed)
        m = build_mlp(DEFAULT_POISSON_MLP).requires_grad_(False)
        if scale != 1.0:
            for p in m.parameters():
                p.mul_(scale)
        return m

    def points(n: int, seed: int = 1):
        g = torch.Generator().manual_seed(seed)
        return torch.rand(n, 2, generator=g) * 2 - 1

    out: dict[str, np.ndarray] = {}
    m0 = model(0)
    m1 = model(1, 3.0)
    out["params_seed0"] = pack_poisson_parameters(m0).numpy()
    out["params_seed1_x3"] = pack_poisson_parameters(m1).numpy()

    for n in FORWARD_BATCHES:
        x = points(n)
        u32, l32 = forward_laplacian(m0, x)
        u64, l64 = forward_laplacian(m0.double(), x.double())
        _, le64 = eager_laplacian(m0.double(), x.double())
        m0.float()
        out[f"fwd{n}_x"] = x.numpy()
        out[f"fwd{n}_u32"] = u32.numpy()
        out[f"fwd{n}_lap32"] = l32.numpy()
        out[f"fwd{n}_u64"] = u64.numpy()
        out[f"fwd{n}_lap64"] = l64.numpy()
        out[f"fwd{n}_eager_lap64"] = le64.detach().numpy()

    xs = points(SATURATED_BATCH)
    u64, l64 = forward_laplacian(m1.double(), xs.double())
    m1.float()
    u32, l32 = forward_laplacian(m1, xs)
    out["sat_x"] = xs.numpy()
    out["sat_u64"], out["sat_lap64"] = u64.numpy(), l64.numpy()
    out["sat_u32"], out["sat_lap32"] = u32.numpy(), l32.numpy()

    def upstream(n: int):
        g = torch.Generator().manual_seed(2)
        return torch.randn(n, 1, generator=g), torch.randn(n, 1, generator=g)

    p0 = pack_poisson_parameters(m0)
    for n in sorted(set(BACKWARD_BATCHES_F32) | set(BACKWARD_BATCHES_F64)):
        x = points(n)
        gu, gl = upstream(n)
        out[f"bwd{n}_x"] = x.numpy()
        out[f"bwd{n}_gu"], out[f"bwd{n}_gl"] = gu.numpy(), gl.numpy()
        if n in BACKWARD_BATCHES_F32:
            gx, gp = _recompute_backward(x, p0, gu, gl, True, True)
            out[f"bwd{n}_gp32"], out[f"bwd{n}_gx32"] = gp.numpy(), gx.numpy()
        if n in BACKWARD_BATCHES_F64:
            gx, gp = _recompute_backward(
                x.double(), p0.double(), gu.double(), gl.double(), True, True
            )
            out[f"bwd{n}_gp64"], out[f"bwd{n}_gx64"] = gp.numpy(), gx.numpy()

    n = SATURATED_BACKWARD_BATCH
    x = points(n)
    gu, gl = upstream(n)
    p1 = pack_poisson_parameters(m1)
    gx, gp = _recompute_backward(x.double(), p1.double(), gu.double(), gl.double(), True, True)
    out["satbwd_x"], out["satbwd_gu"], out["satbwd_gl"] = x.numpy(), gu.numpy(), gl.numpy()
    out["satbwd_gp64"], out["satbwd_gx64"] = gp.numpy(), gx.numpy()

    # Adam trajectory on the interior Poisson loss, through the reference's FL backend.
    train = model(0).requires_grad_(True)
    x = points(ADAM_BATCH)
    source = manufactured_source(x)
    optimizer = torch.optim.Adam(train.parameters(), lr=1e-3, betas=(0.9, 0.999))
    losses = []
    for _ in range(ADAM_STEPS):
        optimizer.zero_grad()
        _, lap = forward_laplacian(train, x)
        loss = (lap - source).pow(2).mean()
        loss.backward()
        optimizer.step()
        losses.append(loss.item())
    out["adam_x"] = x.numpy()
    out["adam_losses"] = np.array(losses, dtype=np.float64)
    out["adam_params_final"] = pack_poisson_parameters(train).detach().numpy()

    # Full PINN loss (interior residual + weighted boundary term) and its gradients.
    from fused_hoad import get_backend
    from fused_hoad.training import boundary_points, poisson_loss_fn

    pinn = model(0).requires_grad_(True)
    xi = points(PINN_INTERIOR)
    xb = boundary_points(PINN_BOUNDARY, device="cpu", generator=torch.Generator().manual_seed(2))
    loss = poisson_loss_fn(get_backend("forward_laplacian"), pinn, xi, xb)()
    loss.backward()
    grads = [torch.cat([pinn[k].weight.grad.reshape(-1), pinn[k].bias.grad.reshape(-1)])
             for k in range(0, len(pinn), 2)]
    out["pinn_x"], out["pinn_xb"] = xi.numpy(), xb.numpy()
    out["pinn_loss"] = np.array(loss.item(), dtype=np.float64)
    out["pinn_grad"] = torch.cat(grads).detach().numpy()

    # SiLU (the reference's other activation: MLPConfig(activation="silu"), models.py:9-12,
    # forward_laplacian.py:34-38). Its fused backend is tanh-only, so the gradients come from
    # autograd through the reference's forward_laplacian on the SiLU model.
    import dataclasses

    silu_config = dataclasses.replace(DEFAULT_POISSON_MLP, activation="silu")

    def silu_model(seed: int, scale: float = 1.0):
        torch.manual_seed(seed)
        m = build_mlp(silu_config).requires_grad_(False)
        if scale != 1.0:
            for p in m.parameters():
                p.mul_(scale)
        return m

    ms = silu_model(0)
    out["silu_params_seed0"] = pack_poisson_parameters(ms).numpy()
    for n in SILU_FORWARD_BATCHES:
        x = points(n)
        u32, l32 = forward_laplacian(ms, x)
        u64, l64 = forward_laplacian(ms.double(), x.double())
        _, le64 = eager_laplacian(ms.double(), x.double())
        ms.float()
        out[f"silufwd{n}_x"] = x.numpy()
        out[f"silufwd{n}_u32"], out[f"silufwd{n}_lap32"] = u32.numpy(), l32.numpy()
        out[f"silufwd{n}_u64"], out[f"silufwd{n}_lap64"] = u64.numpy(), l64.numpy()
        out[f"silufwd{n}_eager_lap64"] = le64.detach().numpy()
    ms3 = silu_model(1, 3.0)
    out["silu_params_seed1_x3"] = pack_poisson_parameters(ms3).numpy()
    xs = points(SATURATED_BATCH)
    u64, l64 = forward_laplacian(ms3.double(), xs.double())
    out["silusat_x"], out["silusat_u64"], out["silusat_lap64"] = xs.numpy(), u64.numpy(), l64.numpy()

    for n in SILU_BACKWARD_BATCHES:
        grad_model = silu_model(0).double().requires_grad_(True)
        x = points(n).double().requires_grad_(True)
        gu, gl = upstream(n)
        u, lap = forward_laplacian(grad_model, x)
        torch.autograd.backward([u, lap], [gu.double(), gl.double()])
        gp = torch.cat([torch.cat([grad_model[k].weight.grad.reshape(-1),
                                   grad_model[k].bias.grad.reshape(-1)])
                        for k in range(0, len(grad_model), 2)])
        out[f"silubwd{n}_x"] = x.detach().float().numpy()
        out[f"silubwd{n}_gu"], out[f"silubwd{n}_gl"] = gu.numpy(), gl.numpy()
        out[f"silubwd{n}_gp64"] = gp.detach().numpy()
        out[f"silubwd{n}_gx64"] = x.grad.detach().numpy()

    train = silu_model(0).requires_grad_(True)
    x = points(ADAM_BATCH)
    source = manufactured_source(x)
    optimizer = torch.optim.Adam(train.parameters(), lr=1e-3, betas=(0.9, 0.999))
    losses = []
    for _ in range(ADAM_STEPS):
        optimizer.zero_grad()
        _, lap = forward_laplacian(train, x)
        loss = (lap - source).pow(2).mean()
        loss.backward()
        optimizer.step()
        losses.append(loss.item())
    out["siluadam_losses"] = np.array(losses, dtype=np.float64)
    out["siluadam_params_final"] = pack_poisson_parameters(train).detach().numpy()

    # The biharmonic: the reference's own higher-order operator, autodiff.laplacian
    # (src/fused_hoad/autodiff.py:39-41), applied to its own output, on the seed-0 MLP
    # (FP32 and FP64) and on the x3 seed-1 MLP (FP64).
    from fused_hoad.autodiff import differentiable_coordinates, laplacian

    def reference_biharmonic(m, x):
        with torch.enable_grad():
            xd = differentiable_coordinates(x)
            u = m(xd)
            lap = laplacian(u, xd)
            bilap = laplacian(lap, xd)
        return u.detach(), lap.detach(), bilap.detach()

    for n in BIHARMONIC_BATCHES:
        x = points(n)
        out[f"bih{n}_x"] = x.numpy()
        for tag in ("32", "64"):  # nn.Module.float()/.double() convert in place
            m = m0.float() if tag == "32" else m0.double()
            u, lap, bilap = reference_biharmonic(m, x if tag == "32" else x.double())
            out[f"bih{n}_u{tag}"] = u.numpy()
            out[f"bih{n}_lap{tag}"] = lap.numpy()
            out[f"bih{n}_bilap{tag}"] = bilap.numpy()
        m0.float()
    xs = points(BIHARMONIC_SATURATED_BATCH)
    u, lap, bilap = reference_biharmonic(m1.double(), xs.double())
    m1.float()
    out["bihsat_x"] = xs.numpy()
    out["bihsat_u64"], out["bihsat_lap64"], out["bihsat_bilap64"] = (
        u.numpy(), lap.numpy(), bilap.numpy())

    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({OUT.stat().st_size / 1024:.0f} KiB, {len(out)} arrays)")


if __name__ == "__main__":
    main()
