"""The bench.py contract on the CPU: the reference arm's JSON line (the same metric, unit,
workload and direction as our arm, with its cpu_baseline and a host-only e2e), the warm-up
rule, and the silent exit of non-zero ranks under torchrun."""

from __future__ import annotations

import importlib.util
import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _bench_module():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def _run(args: list[str], env: dict[str, str] | None = None) -> subprocess.CompletedProcess:
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT,
                          capture_output=True, text=True, timeout=600,
                          env={**os.environ, **(env or {})})


def test_reference_arm_prints_one_contract_line() -> None:
    bench = _bench_module()
    proc = _run(["--impl", "reference", "--steps", "1", "--warmup", "3"])
    assert proc.returncode == 0, proc.stderr
    lines = [ln for ln in proc.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference"
    assert line["metric"] == bench.METRIC and line["unit"] == bench.UNIT
    assert line["higher_is_better"] is True
    assert line["steps"] == 1 and line["warmup"] == 3 and line["n_gpus"] == 1
    assert line["config"]["workload"] == bench.WORKLOAD
    assert line["config"]["points_per_gpu"] == 65_536
    assert line["value"] > 0 and line["ms_per_step"] > 0
    # the reference's published number for this metric (fused fwd v2, 64K points, RTX A5000)
    assert abs(line["vs_baseline"] - line["value"] / bench.PUBLISHED_PTS_S) < 1e-12
    assert "A5000" in line["vs_baseline_note"]
    base = line["cpu_baseline"]
    assert base["kind"] in ("port", "reference") and base["cores"] >= 1
    assert base["value"] == line["value"] and base["unit"] == bench.UNIT and base["sample"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == bench.UNIT
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    # both of the reference's CPU evaluation paths are timed; the line reports the faster
    paths = line["paths"]
    assert set(paths) == {"forward_laplacian", "eager_autograd"}
    assert line["value"] == max(leg["value"] for leg in paths.values())
    assert all(leg["points_per_step"] >= 1024 for leg in paths.values())


def test_warmup_below_three_is_rejected() -> None:
    proc = _run(["--impl", "reference", "--steps", "1", "--warmup", "1"])
    assert proc.returncode != 0
    assert "warmup" in proc.stderr


def test_reference_arm_other_ranks_exit_without_output() -> None:
    proc = _run(["--impl", "reference", "--steps", "1", "--warmup", "3"],
                env={"RANK": "1", "WORLD_SIZE": "2"})
    assert proc.returncode == 0, proc.stderr
    assert proc.stdout.strip() == ""
