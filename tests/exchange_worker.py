"""One rank of the multi-GPU exchange test (run by tests/test_exchange_multigpu.py under
torchrun, one process per GPU).

Every rank trains its shard of one PINN batch twice from the same parameters: with the
in-kernel peer exchange (eager steps, then CUDA-graph replays) and with the NCCL all-reduce
composition. Rank 0 prints one JSON line: whether the peer replicas are bitwise identical
across ranks, the largest difference from the NCCL run, the losses and the status word.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
for entry in (str(ROOT), str(ROOT / "expanded-gpu-optimization_b200")):
    if entry not in sys.path:
        sys.path.insert(0, entry)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import fused_hoad  # noqa: E402
from fused_hoad.distributed import init_from_env, shard_range  # noqa: E402
from oracle import jet  # noqa: E402


def main() -> int:
    rank, world, _ = init_from_env("nccl", timeout_s=60.0)
    C = fused_hoad.load_extension()
    params = jet.init_parameters(0).cuda()
    total, nb = 100_003, 4_001
    x = fused_hoad.uniform_points(total, seed=41).cuda()
    xb = jet.boundary_points(nb, seed=9).cuda()
    a, b = shard_range(total, rank, world)
    c, d = shard_range(nb, rank, world)
    xs, xbs = x[a:b].contiguous(), xb[c:d].contiguous()
    peer = fused_hoad.PoissonTrainer(params.clone(), exchange="peer", wait_limit_s=20.0)
    nccl = fused_hoad.PoissonTrainer(params.clone(), exchange="nccl")
    losses_peer, losses_nccl = [], []
    for _ in range(5):
        losses_peer.append(peer.step(xs, total, boundary=xbs, boundary_total=nb).item())
        losses_nccl.append(nccl.step(xs, total, boundary=xbs, boundary_total=nb).item())
    replay = peer.capture(xs, total, boundary=xbs, boundary_total=nb, warmup=3)
    for _ in range(3):
        nccl.step(xs, total, boundary=xbs, boundary_total=nb)
    for _ in range(10):
        losses_peer.append(replay().item())
        losses_nccl.append(nccl.step(xs, total, boundary=xbs, boundary_total=nb).item())
    torch.cuda.synchronize()
    gathered = [torch.empty_like(peer.params) for _ in range(world)]
    dist.all_gather(gathered, peer.params)
    replicas_equal = all(torch.equal(g, gathered[0]) for g in gathered)
    result = {
        "world": world,
        "replicas_equal": replicas_equal,
        "equal_to_nccl": bool(torch.equal(peer.params, nccl.params)),
        "max_diff_vs_nccl": float((peer.params - nccl.params).abs().max().item()),
        "param_scale": float(nccl.params.abs().max().item()),
        "losses_peer": losses_peer,
        "losses_nccl": losses_nccl,
        "steps": int(peer.step_count.item()),
        "status": int(C.read_device_status(torch.cuda.current_device())),
    }
    del replay  # release the graph before the exchange and the process group
    peer.close()
    dist.barrier()
    if rank == 0:
        print("RESULT " + json.dumps(result), flush=True)
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
