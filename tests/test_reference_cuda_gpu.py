"""Parity with the reference's OWN CUDA kernels, built for sm_100a into oracle/_ref/.

``oracle/build.py`` compiles the reference's three source files unchanged (in the build
container); the library travels to the GPU box with the tree. Skipped when it is absent.
"""

from __future__ import annotations

import importlib.machinery
import importlib.util
from functools import lru_cache

import pytest
import torch
from helpers import assert_scaled

from fused_hoad import fused_forward_laplacian, fused_forward_laplacian_backward, uniform_points
from oracle import jet
from oracle.build import REF_MODULE, ref_library

pytestmark = pytest.mark.gpu


@lru_cache(maxsize=1)
def reference_module():
    path = ref_library()
    if path is None:
        pytest.skip("reference CUDA extension not built (oracle/_ref)")
    loader = importlib.machinery.ExtensionFileLoader(REF_MODULE, str(path))
    spec = importlib.util.spec_from_loader(REF_MODULE, loader)
    module = importlib.util.module_from_spec(spec)
    loader.exec_module(module)
    return module


@pytest.mark.parametrize("version", [0, 1, 2, 3, 4, 5])
@pytest.mark.parametrize("batch", [1, 33, 1_000, 65_536])
def test_forward_matches_reference_fwd_v2(batch: int, version: int) -> None:
    """Every forward version (FP32 CUDA cores 0-2, 3xFP16 3, 3xTF32 4-5) against the
    reference's default FP32 kernel at the reference's tolerance."""
    ref = reference_module()
    params = jet.init_parameters(0).cuda()
    coords = uniform_points(batch, seed=21).cuda()
    ru, rl = ref.fused_forward_laplacian(coords, params, 2)
    u, lap = fused_forward_laplacian(coords, params, version)
    torch.testing.assert_close(u, ru, atol=1e-5, rtol=1e-4)
    torch.testing.assert_close(lap, rl, atol=1e-5, rtol=1e-4)


@pytest.mark.parametrize("batch", [17, 1_000, 65_536])
def test_backward_matches_reference_bwd_v6(batch: int) -> None:
    ref = reference_module()
    params = jet.init_parameters(0).cuda()
    coords = uniform_points(batch, seed=22).cuda()
    g = torch.Generator().manual_seed(5)
    gu = torch.randn(batch, generator=g).cuda()
    gl = torch.randn(batch, generator=g).cuda()
    rp, rx = ref.fused_forward_laplacian_backward(coords, params, gu, gl, 6)
    gp, gx = fused_forward_laplacian_backward(coords, params, gu, gl)
    assert_scaled(gp, rp, 1e-4, "grad params")
    assert_scaled(gx, rx, 1e-4, "grad coords")


def _median_ms(fn, flush, iterations: int = 50) -> float:
    for _ in range(5):
        fn()
    times = []
    for _ in range(iterations):
        flush.zero_()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        fn()
        end.record()
        torch.cuda.synchronize()
        times.append(start.elapsed_time(end))
    times.sort()
    return times[len(times) // 2]


def test_speed_against_reference_kernels() -> None:
    """The reference's own kernels on this GPU are the speed bar (per-call CUDA events,
    median, L2 flushed between calls): our FP32 forward beats its FP32 default (fwd v2), our
    tensor-core forward beats its fastest forward (any version, single TF32 included), and
    our backward beats its default (bwd v6). Prints the table."""
    import json

    ref = reference_module()
    params = jet.init_parameters(0).cuda()
    n = 65_536
    coords = uniform_points(n, seed=1).cuda()
    g = torch.Generator().manual_seed(5)
    gu, gl = torch.randn(n, generator=g).cuda(), torch.randn(n, generator=g).cuda()
    flush = torch.empty(48 << 20, device="cuda")
    rows = {}
    for v in (0, 1, 2, 3, 4, 5):
        rows[f"reference fwd v{v}"] = _median_ms(lambda: ref.fused_forward_laplacian(coords, params, v), flush)
    for v in (0, 1, 2, 3, 4, 5):
        rows[f"ours fwd v{v}"] = _median_ms(lambda: fused_forward_laplacian(coords, params, v), flush)
    for v in (1, 6):
        rows[f"reference bwd v{v}"] = _median_ms(
            lambda: ref.fused_forward_laplacian_backward(coords, params, gu, gl, v), flush)
    rows["ours bwd"] = _median_ms(lambda: fused_forward_laplacian_backward(coords, params, gu, gl), flush)
    table = {k: {"ms": ms, "mpts_per_s": n / ms / 1e3} for k, ms in rows.items()}
    print(json.dumps({"points": n, "gpu": torch.cuda.get_device_name(), "rows": table}, indent=1))
    fastest_reference = min(rows[f"reference fwd v{v}"] for v in range(6))
    assert rows["ours fwd v2"] < rows["reference fwd v2"]
    assert rows["ours fwd v3"] < fastest_reference
    assert rows["ours fwd v4"] < fastest_reference
    assert rows["ours bwd"] < rows["reference bwd v6"]
