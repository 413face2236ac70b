"""Training on the fused kernels: the reference's whole-step CUDA-graph helper and the
B200-native data-parallel Poisson trainer.

``cuda_graph_step`` keeps the reference's signature and behaviour
(``src/fused_hoad/training.py:9-40``) for autograd-based loops over ``fused_laplacian``.

``PoissonTrainer`` is the native step (config: forward jet, backward w.r.t. all 12,737
parameters, Adam at lr 1e-3, betas (0.9, 0.999) on the interior loss
``mean((lap - f)^2)``):

1. one persistent kernel per step recomputes the jet per tile, forms dL/dlap in registers
   and runs the adjoint sweep (no separate forward launch), leaving one partial-gradient
   row per CTA;
2. one update kernel sums the rows in a fixed order, sums over the ranks through the peer
   exchange (``exchange="peer"``, the default: in-kernel over NVLink, no collective launch)
   and applies Adam to the flat parameters in place.

``exchange="nccl"`` runs the same step as separate launches instead -- row reduction into a
flat gradient + loss buffer, one NCCL all-reduce of it, the Adam kernel -- the composition
a library all-reduce gives.

The parameters live in one flat buffer in the reference's ABI, so there is no per-step
pack (``torch.cat``) or gradient split; an ``nn.Module`` handed to the trainer has its
parameters rebound as views of that buffer. The whole step is CUDA-graph capturable.
"""

from __future__ import annotations

from collections.abc import Callable

import torch
from torch import Tensor, nn

from fused_hoad._extension import STATUS_PEER_TIMEOUT, load_extension, read_device_status
from fused_hoad.distributed import PeerExchange, allreduce_sum_, world
from fused_hoad.problem import ACTIVATIONS
from fused_hoad.backends.fused import model_activation
from fused_hoad.parameters import (
    POISSON_PARAMETER_COUNT,
    bind_model_to_flat,
    pack_poisson_parameters,
)


def cuda_graph_step(
    loss_fn: Callable[[], Tensor], optimizer: torch.optim.Optimizer, *, warmup: int = 3
) -> Callable[[], Tensor]:
    """Record one autograd training iteration and return a function that replays it.

    The iteration is ``loss = loss_fn(); loss.backward(); optimizer.step()``. It runs
    ``warmup`` times on a side stream first, so that autograd and the optimizer have set up
    their state before recording. Gradients are then reset to ``None``: the recorded
    backward allocates them again from the graph's private memory pool, so replays reuse
    the same buffers. ``optimizer`` has to be constructed with ``capturable=True`` (its step
    counter then stays on the device). Calling the returned function replays the recorded
    kernels and gives back the loss tensor the recording produced, refreshed in place.
    """
    side_stream = torch.cuda.Stream()
    side_stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side_stream):
        for _ in range(warmup):
            optimizer.zero_grad(set_to_none=True)
            loss_fn().backward()
            optimizer.step()
    torch.cuda.current_stream().wait_stream(side_stream)

    graph = torch.cuda.CUDAGraph()
    optimizer.zero_grad(set_to_none=True)
    with torch.cuda.graph(graph):
        static_loss = loss_fn()
        static_loss.backward()
        optimizer.step()

    def replay() -> Tensor:
        graph.replay()
        return static_loss

    return replay


class PoissonTrainer:
    """Data-parallel Poisson training step on the fused sm_100a kernels.

    ``parameters`` is either the packed 12,737-float CUDA buffer (used in place) or the
    Poisson ``nn.Module``, which is packed once and rebound to views of the buffer.
    With an initialised process group every rank must call :meth:`step` with its own
    shard and the same ``total_points``. ``backward_version`` 6 (default) runs the
    tensor-core step kernel, 1..5 the FP32 CUDA-core one. ``exchange`` picks how the
    gradient is summed over ranks: ``"peer"`` (default) inside the update kernel through
    :class:`PeerExchange` buffers, ``"nccl"`` by an NCCL all-reduce between separate reduction
    and Adam launches. With ``"peer"`` and more than one rank, every rank must construct its
    trainer in the same order and call :meth:`close` after its last step.

    ``activation`` (``"tanh"`` or ``"silu"``) is read from a module, else defaults to tanh;
    SiLU runs the FP32 gradient kernel. The loss is the interior Poisson residual
    ``mean((lap - f)^2)`` (the benchmark's,
    benchmarks/benchmark_training.py:46-48); passing ``boundary`` points to :meth:`step`
    adds the PINN boundary term ``boundary_weight * mean(u^2)`` of the reference's training
    driver (src/fused_hoad/training.py:68-94), in the same kernel launch.

    A peer wait that gives up (a rank that stopped stepping) leaves the affected parameters
    and moments of this rank unchanged for that step, so the replicas would drift apart
    silently; the kernel records it in the device status word instead of hanging.
    :meth:`check_status` reads that word and raises; :meth:`close` calls it, and
    ``check_every=K`` calls it after every K-th eager :meth:`step` (each check synchronises
    the device, so it is skipped inside a stream capture; check after graph replays).
    """

    def __init__(
        self,
        parameters: Tensor | nn.Module,
        *,
        lr: float = 1e-3,
        betas: tuple[float, float] = (0.9, 0.999),
        eps: float = 1e-8,
        group=None,
        backward_version: int = 6,
        boundary_weight: float = 100.0,
        exchange: str = "peer",
        wait_limit_s: float = 30.0,
        activation: str | None = None,
        check_every: int = 0,
    ) -> None:
        self._C = load_extension()
        if check_every < 0:
            raise ValueError("check_every must be >= 0")
        self.check_every = int(check_every)
        self._steps_since_check = 0
        if isinstance(parameters, nn.Module):
            model_act = model_activation(parameters)
            if activation is not None and activation != model_act:
                raise ValueError(f"activation {activation!r} does not match the model's {model_act!r}")
            activation = model_act
            flat = pack_poisson_parameters(parameters).contiguous()
            bind_model_to_flat(parameters, flat)
        else:
            flat = parameters
        self.activation = activation or "tanh"
        if self.activation not in ACTIVATIONS:
            raise ValueError(f"activation must be one of {tuple(ACTIVATIONS)}")
        if not (flat.is_cuda and flat.dtype == torch.float32 and flat.is_contiguous()):
            raise ValueError("parameters must be a contiguous float32 CUDA tensor")
        if flat.numel() != POISSON_PARAMETER_COUNT:
            raise ValueError(f"parameters must have {POISSON_PARAMETER_COUNT} values")
        self.params = flat
        self.exp_avg = torch.zeros_like(flat)
        self.exp_avg_sq = torch.zeros_like(flat)
        self.step_count = torch.zeros(1, dtype=torch.int64, device=flat.device)
        self.lr, self.betas, self.eps = float(lr), (float(betas[0]), float(betas[1])), float(eps)
        self.group = group
        if not 1 <= backward_version <= 6:
            raise ValueError("backward_version must be 1 to 6")
        self.backward_version = int(backward_version)
        self.boundary_weight = float(boundary_weight)
        self._C.prepare_device(flat.device.index if flat.device.index is not None else 0)
        if exchange not in ("peer", "nccl"):
            raise ValueError('exchange must be "peer" or "nccl"')
        self.exchange = exchange
        self._peer = (
            PeerExchange(flat.device, group, wait_limit_s) if exchange == "peer" else None
        )
        self._no_boundary = torch.empty((0, 2), dtype=torch.float32, device=flat.device)

    def check_status(self) -> None:
        """Raise if a bounded wait of this device's kernels gave up since the last read.

        Reads and clears the device status word (synchronises the device). A peer-wait
        timeout means some parameters of this replica missed an update, so training cannot
        continue consistently; any other bit means a kernel returned without its work.
        """
        self._steps_since_check = 0
        status = read_device_status(self.params.device.index or 0)
        if status & STATUS_PEER_TIMEOUT:
            raise RuntimeError(
                "a peer rank's gradient never arrived (exchange wait timed out): this "
                "replica skipped part of an update and no longer matches the others"
            )
        if status:
            raise RuntimeError(f"a kernel's bounded wait gave up (device status {status:#x})")

    def close(self) -> None:
        """Check the device status, then release the peer exchange (collective over the
        group: call on every rank). The exchange is released even when the check raises."""
        if self._peer is None:
            return
        try:
            self.check_status()
        finally:
            self._peer.close()
            self._peer = None

    def _maybe_check(self) -> None:
        if not self.check_every or torch.cuda.is_current_stream_capturing():
            return
        self._steps_since_check += 1
        if self._steps_since_check >= self.check_every:
            self.check_status()

    def gradients(
        self,
        coordinates: Tensor,
        total_points: int,
        boundary: Tensor | None = None,
        boundary_total: int | None = None,
    ) -> Tensor:
        """Flat ``[12738]`` buffer: the gradient summed over ranks, then the loss."""
        if boundary is None:  # the PINN step without a boundary set is the Poisson step
            boundary, boundary_total = self._no_boundary, 0
        elif boundary_total is None:
            boundary_total = boundary.shape[0] * world()[1]
        out = self._C.pinn_step_gradients(
            coordinates, boundary, self.params, total_points, boundary_total,
            self.boundary_weight, self.backward_version, self.activation,
        )
        return allreduce_sum_(out, self.group)

    def step(
        self,
        coordinates: Tensor,
        total_points: int | None = None,
        boundary: Tensor | None = None,
        boundary_total: int | None = None,
    ) -> Tensor:
        """One training step on this rank's points (and boundary points, if given); returns
        the (global) loss, a 1-element device tensor of the loss before the update."""
        if total_points is None:
            total_points = coordinates.shape[0] * world()[1]
        if self.exchange == "peer":
            if self._peer is None:
                raise RuntimeError("trainer is closed")
            if boundary is None:
                boundary, boundary_total = self._no_boundary, 0
            elif boundary_total is None:
                boundary_total = boundary.shape[0] * world()[1]
            loss = self._C.train_step(
                coordinates, boundary, self.params, self.exp_avg, self.exp_avg_sq,
                self.step_count, self.lr, self.betas[0], self.betas[1], self.eps,
                total_points, boundary_total, self.boundary_weight, self._peer.handle,
                self.backward_version, None, self.activation,
            )
            self._maybe_check()
            return loss
        out = self.gradients(coordinates, total_points, boundary, boundary_total)
        self._C.adam_step(
            self.params,
            out[:POISSON_PARAMETER_COUNT],
            self.exp_avg,
            self.exp_avg_sq,
            self.step_count,
            self.lr,
            self.betas[0],
            self.betas[1],
            self.eps,
        )
        self._maybe_check()
        return out[POISSON_PARAMETER_COUNT:]

    def capture(
        self,
        coordinates: Tensor,
        total_points: int | None = None,
        *,
        boundary: Tensor | None = None,
        boundary_total: int | None = None,
        warmup: int = 3,
    ) -> Callable[[], Tensor]:
        """Capture :meth:`step` on ``coordinates`` (and ``boundary``) as one CUDA graph;
        returns ``replay()``.

        The warm-up steps are real steps (they update the parameters). Copy new points into
        ``coordinates`` / ``boundary`` in place between replays.
        """
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self.step(coordinates, total_points, boundary, boundary_total)
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            static_loss = self.step(coordinates, total_points, boundary, boundary_total)

        def replay() -> Tensor:
            graph.replay()
            return static_loss

        replay.graph = graph  # keep alive; release before destroying a process group
        return replay

    def state_dict(self) -> dict[str, Tensor]:
        """Checkpoint: parameters, Adam moments and the step counter."""
        return {
            "params": self.params.detach().clone(),
            "exp_avg": self.exp_avg.clone(),
            "exp_avg_sq": self.exp_avg_sq.clone(),
            "step": self.step_count.clone(),
        }

    def load_state_dict(self, state: dict[str, Tensor]) -> None:
        """Resume from :meth:`state_dict` (copies in place, so captured graphs stay valid)."""
        with torch.no_grad():
            self.params.copy_(state["params"])
            self.exp_avg.copy_(state["exp_avg"])
            self.exp_avg_sq.copy_(state["exp_avg_sq"])
            self.step_count.copy_(state["step"])
