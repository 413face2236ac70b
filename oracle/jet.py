"""PyTorch-on-CPU restatement of the reference's forward-Laplacian oracle (test only).

Every function works on the packed 12,737-float parameter buffer (the ABI of
``csrc/mlp_abi.cuh:8-17`` / ``src/fused_hoad/parameters.py:28-48``) so the same vectors
drive the CUDA kernels and the oracle.

Jet convention (``src/fused_hoad/backends/forward_laplacian.py:3-16``): each hidden state
is ``[batch, dims + 2, width]`` = (value, d/dx_0, d/dx_1, Laplacian). A linear layer is one
matmul with the bias added to the value row only (``:52-57``); tanh applies
``h_v = a, h_J = s z_J, h_L = s z_L - 2 a s |z_J|^2`` with ``a = tanh(z_v), s = 1 - a^2``
(``:28-31, :60-67``); SiLU applies ``h_v = phi, h_J = phi' z_J, h_L = phi' z_L +
phi'' |z_J|^2`` with ``phi = z sigma(z)`` (``:34-38``).
"""

from __future__ import annotations

import math

import torch
from torch import Tensor

INPUTS = 2
HIDDEN = 64
HIDDEN_LAYERS = 4
# (out_features, in_features) per linear layer: src/fused_hoad/parameters.py:29
SHAPES = ((64, 2), (64, 64), (64, 64), (64, 64), (1, 64))
PARAMETER_COUNT = sum(o * i + o for o, i in SHAPES)
assert PARAMETER_COUNT == 12737


def layer_offsets() -> list[tuple[int, int, int, int]]:
    """(weight_offset, bias_offset, out, in) per layer; parameters.py:_make_layout."""
    offsets, offset = [], 0
    for out_features, in_features in SHAPES:
        offsets.append((offset, offset + out_features * in_features, out_features, in_features))
        offset += out_features * in_features + out_features
    return offsets


def unpack(params: Tensor) -> list[tuple[Tensor, Tensor]]:
    """Views ``(W [out, in], b [out])`` into a packed buffer; parameters.py:87-99."""
    if params.ndim != 1 or params.numel() != PARAMETER_COUNT:
        raise ValueError(f"parameters must have shape [{PARAMETER_COUNT}]")
    return [
        (params[w : w + o * i].view(o, i), params[b : b + o])
        for w, b, o, i in layer_offsets()
    ]


def init_parameters(seed: int = 0, scale: float = 1.0, dtype=torch.float32) -> Tensor:
    """Packed parameters of ``torch.manual_seed(seed); build_mlp(DEFAULT_POISSON_MLP)``.

    ``nn.Linear`` default init draws weight then bias per layer, in layer order
    (``src/fused_hoad/models.py:15-26``); building the same modules reproduces the stream.
    """
    torch.manual_seed(seed)
    layers = [torch.nn.Linear(i, o) for o, i in SHAPES]
    with torch.no_grad():
        flat = torch.cat([t.reshape(-1) for layer in layers for t in (layer.weight, layer.bias)])
    return (flat * scale).to(dtype).contiguous()


def uniform_points(n: int, seed: int = 1, dtype=torch.float32) -> Tensor:
    """``torch.rand(n, 2, generator=CPU(seed)) * 2 - 1`` as in the benchmark configs."""
    generator = torch.Generator().manual_seed(seed)
    return (torch.rand(n, 2, generator=generator) * 2 - 1).to(dtype)


def _tanh_jet(jet: Tensor) -> Tensor:
    # forward_laplacian.py:28-31 (_tanh_jet) and :60-67 (_activation)
    z_v, z_j = jet[:, :1], jet[:, 1:-1]
    a = torch.tanh(z_v)
    s = 1.0 - a * a
    out = s * jet
    out[:, -1:].add_(-2.0 * a * s * (z_j * z_j).sum(dim=1, keepdim=True))
    out[:, :1].copy_(a)
    return out


def _silu_jet(jet: Tensor) -> Tensor:
    # forward_laplacian.py:34-38 (_silu_jet) and :60-67 (_activation): phi = z sigma,
    # phi' = sigma (1 + z (1 - sigma)), phi'' = sigma (1 - sigma) (2 + z (1 - 2 sigma))
    z_v, z_j = jet[:, :1], jet[:, 1:-1]
    sigma = torch.sigmoid(z_v)
    first = sigma * (1.0 + z_v * (1.0 - sigma))
    second = sigma * (1.0 - sigma) * (2.0 + z_v * (1.0 - 2.0 * sigma))
    out = first * jet
    out[:, -1:].add_(second * (z_j * z_j).sum(dim=1, keepdim=True))
    out[:, :1].copy_(z_v * sigma)
    return out


# Hidden activations (reference src/fused_hoad/models.py:9-12) and their jets.
ACTIVATION_JETS = {"tanh": _tanh_jet, "silu": _silu_jet}
_ACTIVATION_FNS = {"tanh": torch.tanh, "silu": torch.nn.functional.silu}


def _linear(jet: Tensor, weight: Tensor, bias: Tensor) -> Tensor:
    # forward_laplacian.py:52-57: bias on the value row only
    out = jet @ weight.T
    out[:, 0].add_(bias)
    return out


def forward_laplacian_from_linears(
    linears, coords: Tensor, activation: str = "tanh"
) -> tuple[Tensor, Tensor]:
    """(u, lap) each ``[n, 1]``; forward_laplacian.py:84-92 with :116-132."""
    act_jet = ACTIVATION_JETS[activation]
    n, dims = coords.shape
    jet = coords.new_zeros(n, dims + 2, dims)
    jet[:, 0] = coords
    jet[:, 1:-1] = torch.eye(dims, dtype=coords.dtype, device=coords.device)
    for index, (weight, bias) in enumerate(linears):
        jet = _linear(jet, weight, bias)
        if index < len(linears) - 1:
            jet = act_jet(jet)
    return jet[:, 0], jet[:, -1]


def forward_laplacian(
    params: Tensor, coords: Tensor, activation: str = "tanh"
) -> tuple[Tensor, Tensor]:
    """Forward Laplacian of the packed MLP at ``coords [n, 2]`` in their dtype."""
    return forward_laplacian_from_linears(unpack(params.to(coords.dtype)), coords, activation)


def _eager_laplacian_graph(linears, coords: Tensor, activation: str = "tanh"):
    """(u, lap) by nested autograd, keeping the graph (so lap can be differentiated again
    with respect to the weights); src/fused_hoad/autodiff.py:16-40, reference.py:9-20."""
    x = coords.detach().clone().requires_grad_(True)
    with torch.enable_grad():
        h = x
        for index, (weight, bias) in enumerate(linears):
            h = h @ weight.T + bias
            if index < len(linears) - 1:
                h = _ACTIVATION_FNS[activation](h)
        (first,) = torch.autograd.grad(h.sum(), x, create_graph=True)
        lap = torch.zeros_like(h)
        for d in range(x.shape[1]):
            (second,) = torch.autograd.grad(first[:, d].sum(), x, create_graph=True)
            lap = lap + second[:, d : d + 1]
    return h, lap


def eager_laplacian(
    params: Tensor, coords: Tensor, activation: str = "tanh"
) -> tuple[Tensor, Tensor]:
    """Nested-autograd Laplacian; src/fused_hoad/autodiff.py:16-40, reference.py:9-20."""
    h, lap = _eager_laplacian_graph(unpack(params.to(coords.dtype)), coords, activation)
    return h.detach(), lap.detach()


def cpu_train_step(
    flat: Tensor, coords: Tensor, source: Tensor, optimizer, method: str = "forward_laplacian"
) -> Tensor:
    """One training step of benchmarks/benchmark_training.py:39-57 on the CPU: the Laplacian
    by the forward-Laplacian jet (``method="forward_laplacian"``) or by nested autograd
    (``"eager"``), ``loss = mean((lap - f)^2)``, ``loss.backward()``, ``optimizer.step()``.

    ``flat`` is the packed parameter buffer with ``requires_grad``; the layers are views of
    it, so one backward fills ``flat.grad`` and ``optimizer`` (torch.optim.Adam over
    ``[flat]``) updates all of them. Returns the loss before the update.
    """
    optimizer.zero_grad(set_to_none=True)
    with torch.enable_grad():
        linears = unpack(flat)
        if method == "forward_laplacian":
            _, lap = forward_laplacian_from_linears(linears, coords)
        elif method == "eager":
            _, lap = _eager_laplacian_graph(linears, coords)
        else:
            raise ValueError(f"unknown method {method!r}")
        loss = (lap - source).pow(2).mean()
        loss.backward()
    optimizer.step()
    return loss.detach()


def recompute_backward(
    params: Tensor, coords: Tensor, grad_u: Tensor, grad_lap: Tensor, activation: str = "tanh"
) -> tuple[Tensor, Tensor]:
    """(grad_params [12737], grad_coords [n, 2]); backends/fused.py:76-101.

    Rebuilds the jet from views of the flat buffer and differentiates it with autograd,
    exactly as the reference's ``_recompute_backward`` does.
    """
    dtype = coords.dtype
    with torch.enable_grad():
        x = coords.detach().clone().requires_grad_(True)
        flat = params.detach().to(dtype).clone().requires_grad_(True)
        outputs = forward_laplacian_from_linears(unpack(flat), x, activation)
        grad_x, grad_p = torch.autograd.grad(
            outputs,
            [x, flat],
            (grad_u.reshape(-1, 1).to(dtype), grad_lap.reshape(-1, 1).to(dtype)),
            allow_unused=True,
        )
    if grad_x is None:  # empty batch
        grad_x = torch.zeros_like(coords)
    if grad_p is None:
        grad_p = torch.zeros_like(flat)
    return grad_p.detach(), grad_x.detach()


def manufactured_source(coords: Tensor) -> Tensor:
    """f = -2 pi^2 sin(pi x) sin(pi y); src/fused_hoad/problems/poisson.py:29-39."""
    x, y = coords[:, 0:1], coords[:, 1:2]
    return -2.0 * math.pi**2 * (torch.sin(math.pi * x) * torch.sin(math.pi * y))


def poisson_step_gradients(
    params: Tensor, coords: Tensor, total_points: int | None = None, activation: str = "tanh"
) -> tuple[Tensor, Tensor, Tensor]:
    """Gradients of ``L = sum((lap - f)^2) / total_points`` (benchmark_training.py:46-48).

    ``total_points`` defaults to ``len(coords)`` (the plain mean); a data-parallel shard
    passes the global count so shard gradients sum to the global one. Returns
    ``(loss_partial, grad_params, grad_coords)`` where ``loss_partial`` is this shard's
    contribution to the loss.
    """
    n = coords.shape[0]
    total = n if total_points is None else total_points
    _, lap = forward_laplacian(params, coords, activation)
    residual = lap - manufactured_source(coords)
    loss = (residual * residual).sum() / total
    grad_lap = 2.0 * residual / total
    grad_p, grad_x = recompute_backward(
        params, coords, torch.zeros_like(lap), grad_lap, activation
    )
    return loss, grad_p, grad_x


def boundary_points(count: int, seed: int = 2) -> Tensor:
    """``count`` points uniform on the boundary of [-1, 1]^2 (CPU generator ``seed``): the
    sampling of src/fused_hoad/training.py:45-53 (a side 0..3 for x=-1, x=1, y=-1, y=1,
    a uniform coordinate along it)."""
    g = torch.Generator().manual_seed(seed)
    t = torch.rand(count, generator=g) * 2 - 1
    side = torch.randint(0, 4, (count,), generator=g)
    fixed = torch.where(side % 2 == 0, -1.0, 1.0)
    x_is_fixed = side < 2
    x = torch.where(x_is_fixed, fixed, t)
    y = torch.where(x_is_fixed, t, fixed)
    return torch.stack((x, y), dim=1)


def pinn_step_gradients(
    params: Tensor,
    interior: Tensor,
    boundary: Tensor,
    interior_total: int | None = None,
    boundary_total: int | None = None,
    boundary_weight: float = 100.0,
    activation: str = "tanh",
) -> tuple[Tensor, Tensor]:
    """Gradient of the Poisson PINN loss of src/fused_hoad/training.py:68-94:
    ``sum((lap - f)^2) / interior_total + boundary_weight * sum(u_b^2) / boundary_total``,
    with the totals defaulting to the local counts (plain means). Returns
    ``(loss_partial, grad_params)``; the interior part is ``poisson_step_gradients``, the
    boundary part the VJP of ``u`` alone (grad_u = 2 w u_b / boundary_total, grad_lap = 0).
    """
    nb = boundary.shape[0]
    btotal = nb if boundary_total is None else boundary_total
    loss_i, grad_i, _ = poisson_step_gradients(params, interior, interior_total, activation)
    if nb == 0:
        return loss_i, grad_i
    u_b, _ = forward_laplacian(params, boundary, activation)
    loss_b = boundary_weight * (u_b * u_b).sum() / btotal
    grad_u = 2.0 * boundary_weight * u_b / btotal
    grad_b, _ = recompute_backward(params, boundary, grad_u, torch.zeros_like(u_b), activation)
    return loss_i + loss_b, grad_i + grad_b


def adam_update(
    params: Tensor,
    grad: Tensor,
    exp_avg: Tensor,
    exp_avg_sq: Tensor,
    step: int,
    lr: float = 1e-3,
    beta1: float = 0.9,
    beta2: float = 0.999,
    eps: float = 1e-8,
) -> None:
    """In-place Adam step ``step`` (1-based) with torch.optim.Adam's defaults and formula.

    Restates ``torch.optim.Adam`` (used at benchmarks/benchmark_training.py:41): moments by
    lerp, ``denom = sqrt(v) / sqrt(1 - beta2^t) + eps``, ``p -= lr / (1 - beta1^t) * m / denom``.
    """
    exp_avg.mul_(beta1).add_(grad, alpha=1.0 - beta1)
    exp_avg_sq.mul_(beta2).addcmul_(grad, grad, value=1.0 - beta2)
    bias1 = 1.0 - beta1**step
    bias2 = 1.0 - beta2**step
    denom = exp_avg_sq.sqrt() / math.sqrt(bias2) + eps
    params.addcdiv_(exp_avg, denom, value=-lr / bias1)


# ---- the biharmonic (fourth-order) jet ---------------------------------------------------
#
# Not in the reference, which names the biharmonic as the next operator to test its kernel
# design on (README.md, "Directions to try next"). Its own higher-order tool is nested
# autograd (src/fused_hoad/autodiff.py:39-41, ``laplacian``); ``eager_biharmonic`` applies
# that construction twice and the golden vectors come from the reference's ``laplacian``
# applied twice. The jet carries, per neuron, the nine components
#     [v, g_x, g_y, H_xx, H_xy, H_yy, T_x, T_y, B]
# (value, gradient, Hessian, T = grad(Laplacian), B = biharmonic). A linear layer maps every
# component linearly (the bias only the value); phi = tanh maps them by the chain rule
# (d1..d4 the first to fourth derivatives of tanh at z):
#     H'_ij = d2 g_i g_j + d1 H_ij
#     T'_k  = d3 g_k |g|^2 + 2 d2 (H g)_k + d2 g_k tr H + d1 T_k
#     B'    = d4 |g|^4 + d3 (2 tr H |g|^2 + 4 g.H.g) + d2 (2 |H|_F^2 + 4 g.T + (tr H)^2)
#             + d1 B
# with d1 = 1 - a^2, d2 = -2 a d1, d3 = -2 d1 (1 - 3a^2), d4 = 8 a d1 (2 - 3a^2), a = tanh z.
BIHARMONIC_COMPONENTS = 9


def _tanh_biharmonic_jet(jet: Tensor) -> Tensor:
    """The tanh map of a ``[n, 9, width]`` biharmonic jet (formulas above)."""
    z, gx, gy, hxx, hxy, hyy, tx, ty, b = jet.unbind(1)
    a = torch.tanh(z)
    d1 = 1 - a * a
    d2 = -2 * a * d1
    d3 = -2 * d1 * (1 - 3 * a * a)
    d4 = 8 * a * d1 * (2 - 3 * a * a)
    g2 = gx * gx + gy * gy
    lap = hxx + hyy
    hgx = hxx * gx + hxy * gy
    hgy = hxy * gx + hyy * gy
    ghg = gx * hgx + gy * hgy
    hf2 = hxx * hxx + 2 * hxy * hxy + hyy * hyy
    gt = gx * tx + gy * ty
    return torch.stack(
        (
            a,
            d1 * gx,
            d1 * gy,
            d2 * gx * gx + d1 * hxx,
            d2 * gx * gy + d1 * hxy,
            d2 * gy * gy + d1 * hyy,
            d3 * gx * g2 + 2 * d2 * hgx + d2 * gx * lap + d1 * tx,
            d3 * gy * g2 + 2 * d2 * hgy + d2 * gy * lap + d1 * ty,
            d4 * g2 * g2 + d3 * (2 * lap * g2 + 4 * ghg) + d2 * (2 * hf2 + 4 * gt + lap * lap)
            + d1 * b,
        ),
        dim=1,
    )


def forward_biharmonic(params: Tensor, coords: Tensor) -> tuple[Tensor, Tensor, Tensor]:
    """``(u, lap, bilap)`` each ``[n, 1]`` of the packed tanh MLP by the biharmonic jet, in
    the dtype of ``coords``."""
    linears = unpack(params.to(coords.dtype))
    n = coords.shape[0]
    jet = coords.new_zeros(n, BIHARMONIC_COMPONENTS, 2)
    jet[:, 0] = coords
    jet[:, 1, 0] = 1.0  # d/dx of (x, y)
    jet[:, 2, 1] = 1.0  # d/dy
    for index, (weight, bias) in enumerate(linears):
        jet = jet @ weight.T
        jet[:, 0].add_(bias)
        if index < len(linears) - 1:
            jet = _tanh_biharmonic_jet(jet)
    return jet[:, 0], jet[:, 3] + jet[:, 5], jet[:, 8]


def eager_biharmonic(params: Tensor, coords: Tensor) -> tuple[Tensor, Tensor, Tensor]:
    """``(u, lap, bilap)`` by nested autograd: the Laplacian of the Laplacian, each by the
    construction of src/fused_hoad/autodiff.py:24-41 (the Hessian diagonal, summed)."""
    linears = unpack(params.to(coords.dtype))
    x = coords.detach().clone().requires_grad_(True)

    def laplacian_of(f: Tensor) -> Tensor:
        (first,) = torch.autograd.grad(f.sum(), x, create_graph=True)
        total = torch.zeros_like(f)
        for d in range(x.shape[1]):
            (second,) = torch.autograd.grad(first[:, d].sum(), x, create_graph=True)
            total = total + second[:, d : d + 1]
        return total

    with torch.enable_grad():
        h = x
        for index, (weight, bias) in enumerate(linears):
            h = h @ weight.T + bias
            if index < len(linears) - 1:
                h = torch.tanh(h)
        lap = laplacian_of(h)
        bilap = laplacian_of(lap)
    return h.detach(), lap.detach(), bilap.detach()
