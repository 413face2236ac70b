"""The in-kernel peer exchange across real GPUs: one torchrun rank per GPU
(tests/exchange_worker.py). Skipped with fewer than two GPUs.

Every rank's replica must be bitwise identical to every other's (each rank sums the ranks in
rank order), and the run must follow the NCCL all-reduce composition: bitwise at two ranks
(a sum of two terms has one rounding either way), within 1e-5 of the parameter scale beyond.
"""

from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

WORKER = Path(__file__).resolve().parent / "exchange_worker.py"


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("ranks", [2, 4, 8])
def test_peer_exchange_across_gpus(ranks: int) -> None:
    if torch.cuda.device_count() < ranks:
        pytest.skip(f"needs {ranks} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", OMP_NUM_THREADS="1")
    cmd = [
        "timeout", "-k", "30", "280", sys.executable, "-m", "torch.distributed.run",
        "--nnodes=1", f"--nproc-per-node={ranks}", "--master-addr", "127.0.0.1",
        "--master-port", str(_free_port()), str(WORKER),
    ]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=320)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    line = next(l for l in proc.stdout.splitlines() if l.startswith("RESULT "))
    result = json.loads(line[len("RESULT "):])
    assert result["world"] == ranks
    assert result["status"] == 0
    assert result["steps"] == 18
    assert result["replicas_equal"]
    if ranks == 2:
        assert result["equal_to_nccl"], result["max_diff_vs_nccl"]
    assert result["max_diff_vs_nccl"] <= 1e-5 * result["param_scale"]
    np.testing.assert_allclose(result["losses_peer"], result["losses_nccl"], rtol=1e-5)
