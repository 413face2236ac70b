"""Benchmark of the fused forward-Laplacian hot path (driver contract: one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--points P] [--version V] [--train-steps T]

Headline: residual evaluation ``(u, lap)`` of the
2->64->64->64->64->1 tanh MLP (seed-0 nn.Linear init) at 65,536 uniform points in
[-1,1]^2 per GPU, fp32. A step is one launch of the forward kernel over the rank's points.
With N GPUs (torchrun, one process per GPU) every rank evaluates its own 65,536 points with
no collective (weak scaling) and ``value`` is all ranks' points / the max-over-ranks device
time. Inputs are smaller than L2, so L2 is flushed (a 192 MiB write) between timed steps,
outside the timed events.

Also reported in the same line:
* ``e2e``: the same metric through the public API with host buffers every step: the points
  in pinned host memory, read by the kernel over the host link, (u, lap) written back to
  pinned host memory (``fused_hoad.fused_forward_laplacian_host``); the explicit-copy route
  (H2D copy, ``_C.fused_forward_laplacian``, D2H copies) is reported beside it;
* ``train_step``: BASELINE.json config 2 (fused forward+loss+backward kernel, then one
  update kernel: row reduction, the sum over ranks through the in-kernel NVLink peer
  exchange, Adam) at 65,536 points per GPU; ``--exchange nccl`` times the composition of
  separate launches (row reduction, NCCL all-reduce, Adam) instead;
* ``roofline`` of the forward kernel against the measured peaks in MEASURED_PEAKS.json;
* ``eval_3xtf32``: the same evaluation with forward version 4 (3xTF32, the operand format
  the north star names); ``eval_biharmonic``: (u, lap, bilap) of the same points by the
  biharmonic kernel;
* ``config3``: BASELINE config 3, the evaluation of 1M, 4M and 16M global points split
  evenly over the ranks (strong scaling), per size;
* ``config4``: BASELINE config 4, the training step at 16,777,216 global points (2,097,152 per
  GPU at N=8), graph replay, 100 timed steps by default, with the gradient kernel alone timed
  beside it (the difference is the exchange + Adam), a bitwise all-gather check that every
  rank holds the same parameters and Adam moments, and a 3-step comparison of the in-kernel
  peer exchange with the NCCL all-reduce composition;
* ``cpu_baseline``: the CPU oracle port of the reference's PyTorch paths timed on this host
  (rank 0, N=1 only), a reported baseline: the forward-Laplacian evaluation (``value``), the
  nested-autograd evaluation, both CPU training steps, and both evaluations at 1,024 points.

``--impl reference`` times only the CPU port of the forward-Laplacian evaluation (the
reference's own algorithm; the reference package itself does not exist on the GPU box) on
the same metric and prints its line.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT), str(ROOT / "expanded-gpu-optimization_b200")]

import torch  # noqa: E402

METRIC = "collocation pts/sec for (u,Δu) eval and fwd+bwd step at 64K–16M pts, 1–8 GPU"
UNIT = "pts/s"
FLOP_FORWARD = 101_888  # per point: 3 hidden 64x64 jet GEMMs x 4 comps + layer 0/out + tanh jet
FLOP_STEP = 98_304 * 3 + 256 * 2 + 6_000  # forward + input adjoint + weight gradient + small
# per point: 3 hidden 64x64 GEMMs x 9 jet components, layer 0 and the 3-output layer, and
# about 45 flops of the nine-component tanh map per neuron (256 neurons)
FLOP_BIHARMONIC = 3 * 64 * 64 * 9 * 2 + 640 + 256 * 45
POINTS_PER_GPU = 65_536
CONFIG3_POINTS = (1_048_576, 4_194_304, 16_777_216)  # global points, split over the ranks
CONFIG4_POINTS = 16_777_216                          # global points per training step
WORKLOAD = "config1: residual eval (u, lap) of the 2->64->64->64->64->1 tanh MLP"
# The reference's only published number for this metric: fused fwd v2 (its default) at
# 65,536 points, 0.538 ms = 121.9 M pts/s on an RTX A5000 (reference
# results/2026-11-06-RTX-A5000-8454035/inference.txt:47, README.md:63). It publishes no B200,
# multi-GPU or larger-N numbers.
PUBLISHED_PTS_S = 121.9e6
PUBLISHED_NOTE = ("value / 121.9 M pts/s, the reference's published fused fwd v2 at 65,536 "
                  "points on an RTX A5000 (its only published hardware)")
F16_TRAFFIC = 626_688  # DRAM bytes of one version-3 launch at 65,536 points (ncu)
TF32_TRAFFIC = 632_576  # the same for version 4 (3xTF32)
FLUSH_BYTES = 192 << 20
PEAKS_FILE = ROOT / "MEASURED_PEAKS.json"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
                  "sm_max_mhz": 1965.0}
SM_COUNT = 148
CLOCK_QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
               "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
               "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    p.add_argument("--gpus", type=int, default=int(os.environ.get("WORLD_SIZE", "1")))
    p.add_argument("--steps", type=int, default=3000)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--points", type=int, default=POINTS_PER_GPU, help="points per GPU")
    p.add_argument("--version", type=int, default=None, help="forward kernel version")
    p.add_argument("--train-steps", type=int, default=None)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                   help="how the training step sums gradients over ranks")
    p.add_argument("--activation", choices=["tanh", "silu"], default="tanh",
                   help="hidden activation (the BASELINE configs use tanh)")
    p.add_argument("--config3-steps", type=int, default=20,
                   help="timed evaluations per config-3 size (0 skips the leg)")
    p.add_argument("--config4-steps", type=int, default=100,
                   help="timed training steps of config 4 (0 skips the leg)")
    return p.parse_args()


def load_peaks() -> tuple[dict, str]:
    if PEAKS_FILE.exists():
        return json.loads(PEAKS_FILE.read_text()), "measured"
    return FALLBACK_PEAKS, "fallback"


# ------------------------------------------------------------------ clocks ----

class ClockSampler:
    """nvidia-smi sampling of this rank's GPU while the timed region runs."""

    def __init__(self, gpu_index: int):
        # nvidia-smi numbers GPUs physically; map through CUDA_VISIBLE_DEVICES when set
        visible = [v.strip() for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
        self.gpu = visible[gpu_index] if gpu_index < len(visible) else gpu_index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={CLOCK_QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is None:
            return False
        time.sleep(0.1)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        self.lines = [line for line in out.splitlines() if line.strip()]
        return False

    def summary(self) -> dict:
        sm, mx, reasons, power = [], 0.0, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
                power.append(float(f[3]))
            except ValueError:
                continue
            for name, flag in zip(names, f[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": mx or None,
            "reasons": sorted(reasons),
            "samples": len(sm),
            "power_w_max": max(power) if power else None,
        }


# ---------------------------------------------------------- CPU baseline ----

def _time_cpu_leg(run, budget_s: float, min_runs: int = 3) -> tuple[float, int]:
    """Median seconds per call of `run` after two warm-up calls, calling until `budget_s`
    has passed and at least `min_runs` calls were made (benchmarks/timing.py:40-46)."""
    run()
    run()
    times = []
    deadline = time.perf_counter() + budget_s
    while len(times) < min_runs or time.perf_counter() < deadline:
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
        if len(times) >= 1000:
            break
    return statistics.median(times), len(times)


def cpu_baseline(points: int, budget_s: float, steps: int | None = None) -> dict:
    """The oracle port of the reference's PyTorch paths timed on this host's cores.

    ``value`` is the forward-Laplacian evaluation of the rank's workload (the headline's
    metric); ``legs`` adds the nested-autograd evaluation, both CPU training steps
    (benchmarks/benchmark_training.py:39-57: Laplacian, mean squared residual, backward,
    torch.optim.Adam) at the same size, and both evaluations at config 0's 1,024 points.
    Each leg is the median of its calls within about budget_s / 6 seconds (3 calls at least,
    after 2 warm-up calls)."""
    from oracle import jet

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    params = jet.init_parameters(0)
    leg_budget = budget_s / 6.0
    legs = []

    def add_leg(name: str, n: int, run) -> float:
        sec, calls = _time_cpu_leg(run, leg_budget)
        legs.append({"leg": name, "points": n, "value": n / sec, "unit": UNIT,
                     "ms_per_call": sec * 1e3, "calls": calls})
        return n / sec

    coords = jet.uniform_points(points)
    value = add_leg("forward-Laplacian eval", points, lambda: jet.forward_laplacian(params, coords))
    add_leg("eager (nested autograd) eval", points, lambda: jet.eager_laplacian(params, coords))
    source = jet.manufactured_source(coords)
    for method in ("forward_laplacian", "eager"):
        flat = params.clone().requires_grad_(True)
        optimizer = torch.optim.Adam([flat], lr=1e-3, betas=(0.9, 0.999))
        add_leg(f"{method} train step (loss, backward, Adam)", points,
                lambda: jet.cpu_train_step(flat, coords, source, optimizer, method))
    small = jet.uniform_points(1024)
    add_leg("config0 forward-Laplacian eval", 1024, lambda: jet.forward_laplacian(params, small))
    add_leg("config0 eager eval", 1024, lambda: jet.eager_laplacian(params, small))
    return {
        "value": value,
        "unit": UNIT,
        "cores": cores,
        "kind": "port",
        "sample": (f"forward-Laplacian eval of the {points:,} config-1 points per call, median "
                   f"of {legs[0]['calls']} calls, torch {torch.__version__} on {cores} threads; "
                   "legs: eager eval, both train steps, config 0 (1,024 points)"),
        "ms_per_call": legs[0]["ms_per_call"],
        "legs": legs,
    }


def run_reference(args) -> None:
    """The reference's CPU residual evaluation on all host threads: both of its CPU paths for
    (u, Laplacian u) -- the PyTorch forward-Laplacian jet (backends/forward_laplacian.py) and
    nested eager autograd (autodiff.py) -- each timed over the same bounded sample; the line's
    value is the faster of the two, so the ratio against this arm is against the reference's
    best CPU path on this host."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import jet

    torch.set_num_threads(os.cpu_count() or 1)
    points = args.points
    params = jet.init_parameters(0)
    coords_full = jet.uniform_points(points)
    paths = {"forward_laplacian": jet.forward_laplacian, "eager_autograd": jet.eager_laplacian}
    budget = 60.0  # seconds of timed work per path
    legs = {}
    for name, fn in paths.items():
        probe = coords_full[: min(points, 65536)].contiguous()
        fn(params, probe)
        t0 = time.perf_counter()
        fn(params, probe)
        per_point = (time.perf_counter() - t0) / probe.shape[0]
        sample = points if args.steps * points * per_point <= budget else max(
            1024, int(budget / (args.steps * per_point)))
        coords = coords_full[:sample].contiguous()
        for _ in range(args.warmup):
            fn(params, coords)
        total = 0.0
        for _ in range(args.steps):
            t = time.perf_counter()
            fn(params, coords)
            total += time.perf_counter() - t
        legs[name] = {"value": sample * args.steps / total, "points_per_step": sample,
                      "ms_per_step": total / args.steps * 1e3}
    best = max(legs, key=lambda k: legs[k]["value"])
    value = legs[best]["value"]
    sample = legs[best]["points_per_step"]
    cores = os.cpu_count() or 1
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": legs[best]["ms_per_step"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": value / PUBLISHED_PTS_S,
        "vs_baseline_note": PUBLISHED_NOTE, "dtype": "f32",
        "data": "synthetic (uniform points in [-1,1]^2, CPU generator seed 1; seed-0 nn.Linear init)",
        "config": {"workload": WORKLOAD, "points_per_gpu": points, "global_points": points,
                   "points_per_step": sample, "parallelism": "rank 0 only (CPU)"},
        "impl": "reference",
        "paths": legs,
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"{sample:,} points per step of the {points:,}-point "
                                   f"workload; the faster ({best}) of the reference's two CPU "
                                   f"paths, PyTorch forward Laplacian (oracle port of "
                                   f"src/fused_hoad/backends/forward_laplacian.py) and nested "
                                   f"eager autograd (src/fused_hoad/autodiff.py), on {cores} "
                                   f"threads"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------- our arm ----

def run_ours(args) -> None:
    import torch.distributed as dist

    import fused_hoad
    from fused_hoad.distributed import init_from_env

    rank, world, local_rank = init_from_env("nccl")
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    C = fused_hoad.load_extension()
    C.prepare_device(local_rank)
    version = args.version if args.version is not None else 3
    act = args.activation
    n = args.points
    params = fused_hoad.pack_poisson_parameters(
        (torch.manual_seed(0), fused_hoad.build_mlp())[1]
    ).to(device)
    # each rank's shard: points [rank*n, (rank+1)*n) of the global uniform set
    host = fused_hoad.uniform_points(n * world, seed=1)[rank * n:(rank + 1) * n].contiguous()
    coords = host.to(device)
    flush = torch.empty(FLUSH_BYTES // 4, device=device)
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-timed eval (headline) ----
    # The clock sampler starts first (it waits 0.3 s for nvidia-smi): the warm-up steps then
    # run right before the timed ones, so the first timed launch does not find an idle GPU
    # (measured: the first launch after the GPU sat idle takes 52-82 us instead of 43 us).
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
    with ClockSampler(local_rank) as clocks:
        for _ in range(args.warmup):
            C.fused_forward_laplacian(coords, params, version, act)
            flush.zero_()
        barrier()
        for start, end in events:
            flush.zero_()
            start.record(stream)
            C.fused_forward_laplacian(coords, params, version, act)
            end.record(stream)
        barrier()
    eval_ms = [s.elapsed_time(e) for s, e in events]
    total_ms = max_over_ranks(sum(eval_ms))
    ms_per_step = total_ms / args.steps
    value = n * world * args.steps / (total_ms / 1e3)

    # ---- e2e: host buffers in, host buffers out, every step inside the timed region ----
    pinned_in = host.pin_memory()
    pinned_u = torch.empty(n, 1).pin_memory()
    pinned_lap = torch.empty(n, 1).pin_memory()
    e2e_steps = max(1, min(args.steps, 1000))
    dev_in = torch.empty_like(coords)

    def staged_step():  # explicit H2D copy, kernel, D2H copies
        dev_in.copy_(pinned_in, non_blocking=True)
        u, lap = C.fused_forward_laplacian(dev_in, params, version, act)
        pinned_u.copy_(u, non_blocking=True)
        pinned_lap.copy_(lap, non_blocking=True)

    def zero_copy_step():  # the kernel reads/writes the pinned host buffers directly
        fused_hoad.fused_forward_laplacian_host(pinned_in, params, version, pinned_u, pinned_lap,
                                                act)

    def time_e2e(step) -> float:
        for _ in range(max(3, args.warmup)):
            step()
            flush.zero_()
        events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(e2e_steps)]
        barrier()
        for start, end in events:
            flush.zero_()
            start.record(stream)
            step()
            end.record(stream)
        barrier()
        total = max_over_ranks(sum(s.elapsed_time(e) for s, e in events))
        return n * world * e2e_steps / (total / 1e3)

    reference_lap = C.fused_forward_laplacian(coords, params, version, act)[1].cpu()
    staged_value = time_e2e(staged_step)
    staged_ok = torch.equal(pinned_lap, reference_lap)
    pinned_lap.zero_()
    e2e_value = time_e2e(zero_copy_step)
    torch.cuda.synchronize()
    ok = torch.equal(pinned_lap, reference_lap) and staged_ok

    # ---- the 3xTF32 forward (versions 4/5, the operand format north_star names) ----
    tf32_ms = None
    if version != 4:
        tf32_steps = max(1, min(args.steps, 1000))
        for _ in range(3):
            C.fused_forward_laplacian(coords, params, 4, act)
            flush.zero_()
        events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(tf32_steps)]
        barrier()
        for start, end in events:
            flush.zero_()
            start.record(stream)
            C.fused_forward_laplacian(coords, params, 4, act)
            end.record(stream)
        barrier()
        tf32_ms = max_over_ranks(sum(s.elapsed_time(e) for s, e in events)) / tf32_steps

    # ---- the biharmonic (u, lap, bilap) on the FP32 CUDA cores, same points ----
    bih_steps = max(1, min(args.steps, 500))
    for _ in range(3):
        C.fused_forward_biharmonic(coords, params)
        flush.zero_()
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(bih_steps)]
    barrier()
    for start, end in events:
        flush.zero_()
        start.record(stream)
        C.fused_forward_biharmonic(coords, params)
        end.record(stream)
    barrier()
    bih_ms = max_over_ranks(sum(s.elapsed_time(e) for s, e in events)) / bih_steps

    # ---- training step (config 2) ----
    # One step = weight pre-split, fused forward+loss+backward kernel, update kernel (row
    # reduction + sum over ranks through peer memory + Adam); with --exchange nccl the update
    # is row reduction, [NCCL all-reduce,] Adam. Timed as a CUDA-graph replay (the step's
    # launches replayed without host round trips), and eagerly through PoissonTrainer.step.
    train_steps = args.train_steps if args.train_steps is not None else max(50, args.steps // 10)

    def time_runs(run, count: int) -> float:
        """Sum over `count` calls of `run` of the device time between events bracketing each
        call (L2 flushed before each, outside the events), max over ranks, in ms."""
        events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(count)]
        barrier()
        for start, end in events:
            flush.zero_()
            start.record(stream)
            run()
            end.record(stream)
        barrier()
        return max_over_ranks(sum(s.elapsed_time(e) for s, e in events))

    trainer = fused_hoad.PoissonTrainer(params.clone(), exchange=args.exchange, activation=act)
    for _ in range(max(3, args.warmup)):
        trainer.step(coords, n * world)
    eager_total = time_runs(lambda: trainer.step(coords, n * world), train_steps)
    train_mode = "cuda_graph"
    replay = None
    try:
        replay = trainer.capture(coords, n * world, warmup=3)
        train_total = time_runs(replay, train_steps)
    except RuntimeError as exc:  # capture unavailable: report the eager number
        train_mode = f"eager (graph capture failed: {str(exc).splitlines()[0][:120]})"
        train_total = eager_total
    loss = replay() if replay is not None else trainer.step(coords, n * world)
    final_loss = float(loss.item())
    if replay is not None:
        del replay.graph  # release the captured graph (and any collective in it)
        replay = None
    trainer.close()  # collective over the ranks with the peer exchange
    train_ms = train_total / train_steps
    train_value = n * world * train_steps / (train_total / 1e3)
    eager_value = n * world * train_steps / (eager_total / 1e3)

    # ---- config 3: evaluation of 1M / 4M / 16M global points split over the ranks ----
    config3 = None
    if args.config3_steps > 0:
        config3 = run_config3(args, C, params, version, act, rank, world, device, time_runs)

    # ---- config 4: 16M global points per training step, 100 graph-replayed steps ----
    config4 = None
    if args.config4_steps > 0:
        config4 = run_config4(args, C, params, act, rank, world, device, time_runs)

    peaks, peak_kind = load_peaks()
    clk = clocks.summary()
    if rank != 0:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return

    # DRAM read + write bytes of one forward launch at 65,536 points, from one ncu capture of
    # the same command per kernel family (0-2: FP32 kernel, 3: 3xFP16, 4-5: 3xTF32).
    traffic = None
    if n == POINTS_PER_GPU and act == "tanh":
        traffic = {0: 611_840, 1: 611_840, 2: 611_840, 3: F16_TRAFFIC, 4: TF32_TRAFFIC,
                   5: TF32_TRAFFIC}[version]
    per_launch_s = ms_per_step / 1e3
    achieved_tflops = n * FLOP_FORWARD / per_launch_s / 1e12
    fp32_peak = SM_COUNT * 128 * 2 * peaks.get("sm_max_mhz", 1965.0) * 1e6 / 1e12
    if version <= 2:
        roofline = {
            "bound": "fp32", "achieved": achieved_tflops, "peak": fp32_peak, "unit": "TFLOP/s",
            "frac": achieved_tflops / fp32_peak, "traffic": traffic,
            "kernel": f"forward_fp32_kernel (version {version})",
            "peak_note": ("FP32 CUDA-core peak 148 SMs x 128 lanes x 2 x sm_max_mhz "
                          f"({peak_kind} sm_max_mhz); no measured FP32 peak exists"),
            "flop_per_point": FLOP_FORWARD,
        }
    else:
        bf16 = peaks["bf16_tflops"]
        f16 = version == 3 and act == "tanh"  # SiLU runs the 3xTF32 format
        roofline = {
            "bound": "tensor", "achieved": achieved_tflops, "peak": bf16, "unit": "TFLOP/s",
            "frac": achieved_tflops / bf16, "traffic": traffic,
            "kernel": ("forward_tc_kernel<true> (version 3, 3xFP16)" if f16 else
                       f"forward_tc_kernel<false> (version {version}, 3xTF32)"),
            "peak_note": (f"{peak_kind} bf16 burst peak. Each algorithmic product costs three "
                          "MMAs (hi.hi, lo.hi, hi.lo); f16 runs at the bf16 rate and tf32 at "
                          "half of it, so the split ceiling is bf16/3 for 3xFP16 and bf16/6 "
                          "for 3xTF32"),
            "split_ceiling": bf16 / (3.0 if f16 else 6.0),
            "frac_of_split_ceiling": achieved_tflops / (bf16 / (3.0 if f16 else 6.0)),
            "flop_per_point": FLOP_FORWARD,
        }
    if clk["sm_mhz"]:
        roofline["fp32_peak_at_median_clock"] = SM_COUNT * 256 * clk["sm_mhz"] * 1e6 / 1e12

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": value / PUBLISHED_PTS_S,
        "vs_baseline_note": PUBLISHED_NOTE, "dtype": "f32",
        "data": "synthetic (uniform points in [-1,1]^2, CPU generator seed 1; seed-0 nn.Linear init)",
        "config": {
            "workload": WORKLOAD,
            "points_per_gpu": n, "global_points": n * world, "forward_version": version,
            "activation": act,
            "l2": f"flushed between timed steps ({FLUSH_BYTES >> 20} MiB write, outside the events)",
            "parallelism": f"dp{world}",
        },
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": n * 8,
                "d2h_bytes_per_step": n * 8, "steps": e2e_steps,
                "api": "fused_hoad.fused_forward_laplacian_host (pinned host in/out, the "
                       "kernel moves the bytes over the host link while it computes)",
                "staged_copies_value": staged_value,
                "staged_copies_api": "H2D copy + fused_hoad._C.fused_forward_laplacian + D2H",
                "result_checked": ok},
        "gpu_launches": args.steps,
        "roofline": roofline,
        "clocks": clk,
        "eval_3xtf32": None if tf32_ms is None else {
            "kernel": "forward_tc_kernel<false> (version 4, 3xTF32)",
            "value": n * world / (tf32_ms / 1e3), "unit": UNIT, "ms_per_step": tf32_ms,
            "achieved_tflops": n * FLOP_FORWARD / (tf32_ms / 1e3) / 1e12,
            "frac_of_split_ceiling": (n * FLOP_FORWARD / (tf32_ms / 1e3) / 1e12)
                                     / (peaks["bf16_tflops"] / 6.0),
        },
        "eval_biharmonic": {
            "kernel": "forward_biharmonic_kernel (FP32 CUDA cores, nine-component jet)",
            "outputs": "u, Laplacian, biharmonic", "points_per_gpu": n,
            "value": n * world / (bih_ms / 1e3), "unit": UNIT, "ms_per_step": bih_ms,
            "steps": bih_steps, "flop_per_point": FLOP_BIHARMONIC,
            "achieved_tflops": n * FLOP_BIHARMONIC / (bih_ms / 1e3) / 1e12,
            "frac_of_fp32_peak": (n * FLOP_BIHARMONIC / (bih_ms / 1e3) / 1e12) / fp32_peak,
        },
        "train_step": {
            "workload": "config2: fused forward+loss+backward kernel, " + (
                "update kernel (row reduction, "
                + ("sum over ranks through NVLink peer memory, " if world > 1 else "")
                + "Adam)" if args.exchange == "peer" else
                "row reduction, " + ("NCCL all-reduce, " if world > 1 else "") + "fused Adam"),
            "exchange": args.exchange,
            "value": train_value, "unit": UNIT, "ms_per_step": train_ms, "steps": train_steps,
            "timing": train_mode, "eager_value": eager_value,
            "backward_kernel": ("backward_tc_kernel (version 6)" if act == "tanh" else
                                "backward_fp32_kernel (SiLU: every version)"),
            "points_per_gpu": n,
            "launches_per_step": 3 if args.exchange == "peer" else 4 + (1 if world > 1 else 0),
            "loss_after": final_loss,
            "achieved_tflops": n * FLOP_STEP / (train_ms / 1e3) / 1e12,
            "flop_per_point": FLOP_STEP,
        },
        "config3": config3,
        "config4": config4,
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(n, budget_s=24.0)
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_config3(args, C, params, version, act, rank, world, device, time_runs) -> dict:
    """(u, lap) of 1M, 4M and 16M global uniform points, each split evenly
    by index over the ranks (strong scaling: the global count is fixed as N grows).
    ``value`` per size = global points / the max-over-ranks device time of one evaluation."""
    import fused_hoad

    host = fused_hoad.uniform_points(max(CONFIG3_POINTS), seed=1)
    sizes = []
    for total in CONFIG3_POINTS:
        a, b = fused_hoad.shard_range(total, rank, world)
        shard = host[a:b].to(device)
        for _ in range(3):
            C.fused_forward_laplacian(shard, params, version, act)
        total_ms = time_runs(lambda: C.fused_forward_laplacian(shard, params, version, act),
                             args.config3_steps)
        ms = total_ms / args.config3_steps
        sizes.append({"global_points": total, "points_per_gpu": b - a,
                      "value": total / (ms / 1e3), "unit": UNIT, "ms_per_step": ms,
                      "steps": args.config3_steps})
        del shard
    return {"workload": "config3: residual eval (u, lap) at 1M/4M/16M global points, split "
                        "evenly by point index over the ranks",
            "forward_version": version, "scaling": "strong", "sizes": sizes,
            "points": "the first 1M/4M/16M rows of one 16,777,216-point uniform draw (seed 1)"}


def run_config4(args, C, params, act, rank, world, device, time_runs) -> dict:
    """data-parallel Poisson training at 16,777,216 global points per step
    (16M / N per rank), graph-replayed steps (gradient kernel, then the update kernel that
    sums over the ranks and applies Adam), then a bitwise cross-rank check of the replicas.

    ``gradients_only_ms`` times the same gradient kernel plus a local fixed-order row
    reduction without the exchange and Adam; ``update_overhead_ms`` = step - that, the cost
    of the cross-rank sum (including the wait for the slowest rank) and Adam."""
    import torch.distributed as dist

    import fused_hoad

    total = CONFIG4_POINTS
    a, b = fused_hoad.shard_range(total, rank, world)
    coords = fused_hoad.uniform_points(total, seed=1)[a:b].to(device)
    trainer = fused_hoad.PoissonTrainer(params.clone(), exchange=args.exchange, activation=act)
    replay = trainer.capture(coords, total, warmup=3)
    step_total = time_runs(replay, args.config4_steps)
    steps_done = int(trainer.step_count.item())
    loss = float(replay().item())
    del replay.graph
    replay = None
    trainer.check_status()

    def gathered_equal(t: torch.Tensor) -> bool:
        if world == 1:
            return True
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t.contiguous())
        return all(torch.equal(q, parts[0]) for q in parts)

    replicas_equal = all(gathered_equal(t) for t in
                         (trainer.params, trainer.exp_avg, trainer.exp_avg_sq,
                          trainer.step_count))
    trainer.close()

    # gradient kernel + local row reduction alone (no exchange, no Adam), same shard
    for _ in range(3):
        C.poisson_step_gradients(coords, params, total)
    grad_total = time_runs(lambda: C.poisson_step_gradients(coords, params, total),
                           args.config4_steps)

    # the in-kernel peer exchange against the NCCL all-reduce composition, from one start
    peer = fused_hoad.PoissonTrainer(params.clone(), exchange="peer", activation=act)
    nccl = fused_hoad.PoissonTrainer(params.clone(), exchange="nccl", activation=act)
    for _ in range(3):
        peer.step(coords, total)
        nccl.step(coords, total)
    torch.cuda.synchronize()
    equal_to_nccl = bool(torch.equal(peer.params, nccl.params))
    max_diff = float((peer.params - nccl.params).abs().max().item())
    scale = float(nccl.params.abs().max().item())
    peer.close()

    ms = step_total / args.config4_steps
    grad_ms = grad_total / args.config4_steps
    return {
        "workload": "config4: Poisson training step at 16,777,216 global points (fused "
                    "forward+loss+backward kernel, update kernel: row sums, the sum over "
                    "ranks, Adam), CUDA-graph replay",
        "exchange": args.exchange, "scaling": "strong", "global_points": total,
        "points_per_gpu": b - a, "steps": args.config4_steps,
        "value": total / (ms / 1e3), "unit": UNIT, "ms_per_step": ms,
        "achieved_tflops_per_gpu": (b - a) * FLOP_STEP / (ms / 1e3) / 1e12,
        "gradients_only_ms": grad_ms, "update_overhead_ms": ms - grad_ms,
        "update_overhead_share": (ms - grad_ms) / ms,
        "loss_after": loss, "steps_applied": steps_done,
        "replicas_equal": replicas_equal,
        "replicas_check": "all_gather of params, exp_avg, exp_avg_sq and the step counter "
                          "after the timed steps; torch.equal against rank 0's (bitwise)",
        "peer_vs_nccl": {"steps": 3, "equal": equal_to_nccl, "max_abs_diff": max_diff,
                         "param_scale": scale,
                         "note": "bitwise equal expected at N <= 2 (a sum of two values does "
                                 "not depend on order); NCCL's order differs beyond"},
    }


def main() -> None:
    args = parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
