"""Data-parallel plumbing: one process per GPU, collocation points sharded by index.

Every point is independent, so a batch splits into contiguous index ranges, one per rank
(``shard_range``). Evaluation needs no collective at all. Training needs exactly one: the
sum of the flat gradient (12,737 floats, plus the loss in one extra slot) over ranks,
after which every rank applies the identical fused Adam update to its replica, so no
broadcast is needed. The reference has no multi-GPU path; this module is the new part.

Two ways to do that sum: ``PeerExchange`` (the default of the trainer) does it inside the
step's update kernel, through buffers every rank maps from every other over NVLink (CUDA
IPC), so the step has no collective launch; ``allreduce_sum_`` is one NCCL all-reduce.
"""

from __future__ import annotations

import os
from datetime import timedelta

import torch
import torch.distributed as dist


def shard_range(total: int, rank: int, world_size: int) -> tuple[int, int]:
    """``[start, stop)`` of rank ``rank``'s contiguous shard of ``total`` points.

    Shards differ in size by at most one point; the first ``total % world_size`` ranks
    take the extra points.
    """
    if world_size < 1 or not 0 <= rank < world_size or total < 0:
        raise ValueError("need world_size >= 1, 0 <= rank < world_size, total >= 0")
    base, extra = divmod(total, world_size)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def world() -> tuple[int, int]:
    """``(rank, world_size)`` of the default group, ``(0, 1)`` when not initialised."""
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


def init_from_env(backend: str = "nccl", timeout_s: float = 120.0) -> tuple[int, int, int]:
    """Initialise the default process group from torchrun's environment variables.

    Returns ``(rank, world_size, local_rank)``; binds this process to GPU ``local_rank``
    when the backend is NCCL. Without ``WORLD_SIZE`` > 1 nothing is initialised.
    """
    world_size = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world_size <= 1:
        return 0, 1, local_rank
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    if backend == "nccl":
        torch.cuda.set_device(local_rank)
    kwargs = {}
    if backend == "nccl":
        kwargs["device_id"] = torch.device("cuda", local_rank)
    dist.init_process_group(
        backend=backend,
        rank=rank,
        world_size=world_size,
        timeout=timedelta(seconds=timeout_s),
        **kwargs,
    )
    return rank, world_size, local_rank


def allreduce_sum_(tensor: torch.Tensor, group=None) -> torch.Tensor:
    """In-place sum over the ranks of ``group`` (a no-op on one rank)."""
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(tensor, op=dist.ReduceOp.SUM, group=group)
    return tensor


class PeerExchange:
    """This rank's side of the in-kernel gradient exchange of the fused training step.

    Every rank of ``group`` (the default group when None; a single rank without one) creates
    one on its own GPU, in the same order: the ranks share their buffers' CUDA IPC handles
    through ``group`` (``all_gather_object``) and map each other's. Each training step then
    writes its column sums into every peer's buffer and waits on flags, each wait bounded by
    ``wait_limit_s``; a wait that gives up sets ``FHB_STATUS_PEER_TIMEOUT`` in the device
    status word (``fused_hoad.read_device_status``). Call :meth:`close` on every rank after
    the last step; it synchronises the device and the group before it frees the buffer.
    """

    def __init__(
        self, device: torch.device | int, group=None, wait_limit_s: float = 30.0
    ) -> None:
        from fused_hoad._extension import load_extension

        self._C = load_extension()
        self.group = group
        if dist.is_available() and dist.is_initialized():
            self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        else:
            self.rank, self.world = 0, 1
        self.device = torch.device("cuda", device) if isinstance(device, int) else device
        index = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self.handle = self._C.exchange_create(self.world, self.rank, float(wait_limit_s), index)
        if self.world > 1:
            mine = bytes(self._C.exchange_handle(self.handle).numpy())
            gathered: list[bytes | None] = [None] * self.world
            dist.all_gather_object(gathered, mine, group=group)
            handles = torch.frombuffer(bytearray(b"".join(gathered)), dtype=torch.uint8)
            self._C.exchange_connect(self.handle, handles)

    def close(self) -> None:
        """Free the exchange (collective over ``group`` when it has more than one rank)."""
        if not self.handle:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        self._C.exchange_destroy(self.handle)
        self.handle = 0
