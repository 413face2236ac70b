"""Data-parallel host logic on CPU ranks (gloo, world_size 2): sharding + the one all-reduce.

The GPU step sums per-shard gradients computed with the global point count; here the
per-shard gradients come from the CPU oracle and go through the same collective glue
(``fused_hoad.distributed``). Also covers failure detection on the host: a rank that never
joins a collective makes the other rank's collective end with an error after a short
process-group timeout (no GPU involved).
"""

from __future__ import annotations

import os
import socket
import traceback
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank: int, world: int, port: int, timeout_s: float) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group(
        "gloo", rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s)
    )


def _sharded_gradient_worker(rank: int, world: int, port: int, results) -> None:
    try:
        import sys
        from pathlib import Path

        root = Path(__file__).resolve().parents[1]
        sys.path[:0] = [str(root), str(root / "expanded-gpu-optimization_b200")]
        from fused_hoad.distributed import allreduce_sum_, shard_range
        from oracle import jet

        torch.set_num_threads(1)
        _init(rank, world, port, 60.0)
        total = 301  # odd: shards differ by one point
        params = jet.init_parameters(0)
        points = jet.uniform_points(total)
        start, stop = shard_range(total, rank, world)
        loss, grad, _ = jet.poisson_step_gradients(params, points[start:stop], total)
        flat = torch.cat([grad, loss.reshape(1)])
        allreduce_sum_(flat)
        if rank == 0:
            full_loss, full_grad, _ = jet.poisson_step_gradients(params, points)
            results.put(
                (
                    float((flat[:-1] - full_grad).abs().max()),
                    float(full_grad.abs().max()),
                    float(flat[-1]),
                    float(full_loss),
                )
            )
        dist.barrier()
        dist.destroy_process_group()
    except Exception:  # pragma: no cover - reported to the parent
        results.put(traceback.format_exc())


def test_sharded_gradients_all_reduce_to_the_full_batch_gradient() -> None:
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sharded_gradient_worker, args=(r, 2, port, results))
             for r in range(2)]
    for p in procs:
        p.start()
    out = results.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert not isinstance(out, str), out
    error, scale, loss, full_loss = out
    assert error <= 1e-5 * scale
    assert abs(loss - full_loss) <= 1e-5 * abs(full_loss)


def _missing_rank_worker(rank: int, world: int, port: int, results) -> None:
    try:
        _init(rank, world, port, 3.0)
        if rank == 1:
            # leaves between steps, without joining the next collective
            results.put("rank1-left")
            return
        try:
            dist.all_reduce(torch.ones(4))
            results.put("no-error")
        except Exception as exc:  # the expected path: the collective times out
            results.put(f"error:{type(exc).__name__}")
    except Exception:  # pragma: no cover
        results.put(traceback.format_exc())


@pytest.mark.timeout(120)
def test_missing_rank_turns_into_a_host_error_not_a_hang() -> None:
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_missing_rank_worker, args=(r, 2, port, results))
             for r in range(2)]
    for p in procs:
        p.start()
    seen = {results.get(timeout=90), results.get(timeout=90)}
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert "rank1-left" in seen
    assert any(s.startswith("error:") for s in seen), seen
