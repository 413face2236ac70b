"""The fused training-step update on one GPU: row sums + exchange + Adam in one kernel.

Checks, against the separate launches it replaces (row reduction, flat-buffer sum, the Adam
kernel) and the oracle:
  * one rank: the fused update gives bitwise the parameters of reduction + Adam;
  * two ranks emulated on one GPU: the test plays rank 1 by writing its epoch-tagged column
    sums into rank 0's exchange buffer before rank 0's step (no second kernel waits on the
    first), and rank 0's own sums must land in rank 1's buffer;
  * a peer that never publishes: the bounded wait gives up, sets FHB_STATUS_PEER_TIMEOUT,
    and the parameters stay unchanged.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch
from helpers import PARAMETER_COUNT, assert_scaled, ptr, read_status, stream_handle

import fused_hoad
from fused_hoad import _native, uniform_points
from oracle import jet

pytestmark = pytest.mark.gpu

ROW = 12740          # FHB_EXCHANGE_ROW_WORDS
MAX_RANKS = 8        # FHB_EXCHANGE_MAX_RANKS
PEER_TIMEOUT = 0x4   # FHB_STATUS_PEER_TIMEOUT


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    read_status()  # start from a clear status word
    yield


class _DeviceWords:
    """A device address seen as a torch int64 tensor (``__cuda_array_interface__``)."""

    def __init__(self, address: int, words: int) -> None:
        self.__cuda_array_interface__ = {
            "shape": (words,), "typestr": "<i8", "data": (address, False), "strides": None,
            "version": 3,
        }


def _buffer_words() -> int:
    return _native.library().fhb_exchange_buffer_bytes() // 8


def _exchange_words(C, handle: int) -> torch.Tensor:
    return torch.as_tensor(_DeviceWords(C.exchange_buffer(handle), _buffer_words()),
                           device="cuda")


def _slot_row(buf: torch.Tensor, epoch: int, source: int) -> torch.Tensor:
    start = ((epoch % 2) * MAX_RANKS + source) * ROW
    return buf[start:start + PARAMETER_COUNT + 1]


def _pack(values: torch.Tensor, epoch: int) -> torch.Tensor:
    """The words a rank stores: epoch in the high half, the float's bits in the low half."""
    return (values.view(torch.int32).to(torch.int64) & 0xFFFFFFFF) | (epoch << 32)


def _epochs(words: torch.Tensor) -> torch.Tensor:
    return words >> 32


def _values(words: torch.Tensor) -> torch.Tensor:
    return (words & 0xFFFFFFFF).to(torch.int32).view(torch.float32)


def _adam_state(params: torch.Tensor):
    return params.clone(), torch.zeros_like(params), torch.zeros_like(params), torch.zeros(
        1, dtype=torch.int64, device=params.device)


HYPER = dict(lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8)


@pytest.mark.parametrize("kernel", [5, 6])
def test_fused_update_is_bitwise_reduction_plus_adam(kernel: int) -> None:
    C = fused_hoad.load_extension()
    params = jet.init_parameters(0).cuda()
    x = uniform_points(20_000, seed=31).cuda()
    xb = jet.boundary_points(1_000, seed=7).cuda()
    ex = C.exchange_create(1, 0, 5.0, 0)
    try:
        p1, m1, v1, s1 = _adam_state(params)
        p2, m2, v2, s2 = _adam_state(params)
        for _ in range(3):
            grad = torch.empty(PARAMETER_COUNT + 1, device="cuda")
            loss = C.train_step(x, xb, p1, m1, v1, s1, HYPER["lr"], HYPER["beta1"],
                                HYPER["beta2"], HYPER["eps"], len(x), len(xb), 100.0, ex,
                                kernel, grad)
            want = C.pinn_step_gradients(x, xb, p2, len(x), len(xb), 100.0, kernel)
            C.adam_step(p2, want[:PARAMETER_COUNT], m2, v2, s2, *HYPER.values())
            assert torch.equal(grad, want)
            assert torch.equal(loss, want[PARAMETER_COUNT:])
        assert torch.equal(p1, p2) and torch.equal(m1, m2) and torch.equal(v1, v2)
        assert int(s1.item()) == 3
    finally:
        C.exchange_destroy(ex)
    assert read_status() == 0


def test_train_step_through_the_c_abi_matches_the_oracle() -> None:
    lib = _native.library()
    params = jet.init_parameters(1).cuda()
    x = uniform_points(4_096, seed=32).cuda()
    p, m, v, step = _adam_state(params)
    handle = ctypes.c_void_p()
    _native.check(lib.fhb_exchange_create(1, 0, 10**9, ctypes.byref(handle)), "create")
    try:
        ws_bytes = lib.fhb_pinn_step_workspace_bytes(len(x), 0)
        ws = torch.empty((ws_bytes + 15) // 16 * 4, device="cuda")
        loss = torch.empty(1, device="cuda")
        for _ in range(2):
            code = lib.fhb_train_step(
                ptr(x), len(x), len(x), None, 0, 0, 100.0, ptr(p), ptr(m), ptr(v), ptr(step),
                1e-3, 0.9, 0.999, 1e-8, handle, None, ptr(loss), 6, 0, ptr(ws), ws_bytes,
                stream_handle())
            _native.check(code, "fhb_train_step")
    finally:
        _native.check(lib.fhb_exchange_destroy(handle), "destroy")
    want_p = params.cpu().clone()
    want_m, want_v = torch.zeros_like(want_p), torch.zeros_like(want_p)
    for t in (1, 2):
        want_loss, grad, _ = jet.poisson_step_gradients(want_p, x.cpu())
        jet.adam_update(want_p, grad, want_m, want_v, t)
    np.testing.assert_allclose(loss.item(), want_loss.item(), rtol=1e-4)
    diff = (p.cpu() - want_p).abs()
    assert float((diff > 1e-5).float().mean()) < 1e-3, float(diff.max())
    # argument checks: a missing exchange and an unconnected one are rejected
    assert lib.fhb_train_step(ptr(x), len(x), len(x), None, 0, 0, 100.0, ptr(p), ptr(m),
                              ptr(v), ptr(step), 1e-3, 0.9, 0.999, 1e-8, None, None,
                              ptr(loss), 6, 0, ptr(ws), ws_bytes, stream_handle()) == 1


@pytest.mark.parametrize("kernel", [5, 6])
def test_two_rank_exchange_emulated_on_one_gpu(kernel: int) -> None:
    """Rank 0 of 2; the test writes rank 1's words, as rank 1's kernel would."""
    C = fused_hoad.load_extension()
    params = jet.init_parameters(2).cuda()
    total = 30_001
    x = uniform_points(total, seed=33).cuda()
    a, b = fused_hoad.shard_range(total, 0, 2)
    x0, x1 = x[a:b].contiguous(), x[b:].contiguous()
    ex = C.exchange_create(2, 0, 5.0, 0)
    peer = torch.zeros(_buffer_words(), dtype=torch.int64, device="cuda")
    try:
        C.exchange_connect_local(ex, [0, peer.data_ptr()])
        own = _exchange_words(C, ex)
        p, m, v, s = _adam_state(params)
        pw, mw, vw, sw = _adam_state(params)
        empty = torch.empty(0, 2, device="cuda")
        for epoch in (1, 2, 3):
            g1 = C.poisson_step_gradients(x1, p, total, version=kernel)[0]
            _slot_row(own, epoch, 1).copy_(_pack(g1, epoch))
            grad = torch.empty(PARAMETER_COUNT + 1, device="cuda")
            loss = C.train_step(x0, empty, p, m, v, s, *HYPER.values(), total, 0, 100.0, ex,
                                kernel, grad)
            g0 = C.poisson_step_gradients(x0, pw, total, version=kernel)[0]
            want = g0 + g1  # rank order: row 0, then row 1
            assert torch.equal(grad, want), epoch
            assert torch.equal(loss, want[PARAMETER_COUNT:])
            C.adam_step(pw, want[:PARAMETER_COUNT], mw, vw, sw, *HYPER.values())
            assert torch.equal(p, pw), epoch
            # rank 0's own sums went into row 0 of both buffers, tagged with the epoch
            for buf in (peer, own):
                assert torch.equal(_values(_slot_row(buf, epoch, 0)), g0)
                assert bool((_epochs(_slot_row(buf, epoch, 0)) == epoch).all())
        # the exchange of two shards is the full-batch step (up to summation order)
        full = C.poisson_step_gradients(x, params, total, version=kernel)[0]
        first = C.poisson_step_gradients(x0, params, total, version=kernel)[0] + \
            C.poisson_step_gradients(x1, params, total, version=kernel)[0]
        assert_scaled(first.cpu(), full.cpu(), 1e-5, "two shards vs full batch")
    finally:
        C.exchange_destroy(ex)
    assert read_status() == 0


def test_peer_that_never_publishes_times_out_without_update() -> None:
    """Rank 1's words never arrive: the bounded wait gives up after 2 ms."""
    C = fused_hoad.load_extension()
    params = jet.init_parameters(3).cuda()
    x = uniform_points(2_048, seed=34).cuda()
    ex = C.exchange_create(2, 0, 0.002, 0)
    peer = torch.zeros(_buffer_words(), dtype=torch.int64, device="cuda")
    try:
        C.exchange_connect_local(ex, [0, peer.data_ptr()])
        p, m, v, s = _adam_state(params)
        C.train_step(x, torch.empty(0, 2, device="cuda"), p, m, v, s, *HYPER.values(),
                     len(x), 0, 100.0, ex, 6)
        torch.cuda.synchronize()
        assert read_status() & PEER_TIMEOUT
        assert torch.equal(p, params) and not m.any() and not v.any()
        # rank 0 still published its words, so a peer would not wait on it
        assert bool((_epochs(_slot_row(peer, 1, 0)) == 1).all())
    finally:
        C.exchange_destroy(ex)
    assert read_status() == 0


def test_trainer_peer_and_nccl_modes_agree_bitwise_on_one_rank() -> None:
    params = jet.init_parameters(4).cuda()
    x = uniform_points(10_000, seed=35).cuda()
    xb = jet.boundary_points(500, seed=8).cuda()
    peer = fused_hoad.PoissonTrainer(params.clone(), exchange="peer")
    nccl = fused_hoad.PoissonTrainer(params.clone(), exchange="nccl")
    for _ in range(4):
        assert torch.equal(peer.step(x, boundary=xb), nccl.step(x, boundary=xb))
    assert torch.equal(peer.params, nccl.params)
    replay = peer.capture(x, boundary=xb, warmup=3)
    for _ in range(3):
        nccl.step(x, boundary=xb)
    for _ in range(5):
        assert torch.equal(replay(), nccl.step(x, boundary=xb))
    assert torch.equal(peer.params, nccl.params)
    assert int(peer.step_count.item()) == int(nccl.step_count.item()) == 12
    peer.close()
    with pytest.raises(RuntimeError, match="closed"):
        peer.step(x)


def test_rank_with_no_points_takes_part_with_zeros() -> None:
    C = fused_hoad.load_extension()
    params = jet.init_parameters(5).cuda()
    ex = C.exchange_create(1, 0, 5.0, 0)
    try:
        p, m, v, s = _adam_state(params)
        grad = torch.full((PARAMETER_COUNT + 1,), float("nan"), device="cuda")
        empty = torch.empty(0, 2, device="cuda")
        C.train_step(empty, empty, p, m, v, s, *HYPER.values(), 10, 0, 100.0, ex, 6, grad)
        assert not grad.any()
        assert torch.equal(p, params)  # Adam with a zero gradient leaves p unchanged
        assert int(s.item()) == 1
    finally:
        C.exchange_destroy(ex)


def test_trainer_raises_when_a_peer_wait_gave_up() -> None:
    """PoissonTrainer turns a peer-wait timeout into an error instead of drifting silently:
    its exchange is swapped for a two-rank one whose rank 1 never publishes (2 ms limit)."""
    C = fused_hoad.load_extension()
    params = jet.init_parameters(3).cuda()
    x = uniform_points(2_048, seed=36).cuda()
    trainer = fused_hoad.PoissonTrainer(params.clone(), exchange="peer", check_every=1)
    own = trainer._peer.handle
    ex = C.exchange_create(2, 0, 0.002, 0)
    peer = torch.zeros(_buffer_words(), dtype=torch.int64, device="cuda")
    try:
        C.exchange_connect_local(ex, [0, peer.data_ptr()])
        trainer._peer.handle = ex
        with pytest.raises(RuntimeError, match="peer rank"):
            trainer.step(x)
        assert torch.equal(trainer.params, params)  # the update was skipped, and reported
    finally:
        trainer._peer.handle = own
        C.exchange_destroy(ex)
    trainer.step(x)  # the trainer's own exchange still works; nothing left to report
    trainer.close()
    assert read_status() == 0


def test_trainer_check_status_reports_any_bounded_wait_bit() -> None:
    lib = _native.library()
    trainer = fused_hoad.PoissonTrainer(jet.init_parameters(0).cuda())
    read_status()
    _native.check(lib.fhb_debug_bounded_wait_selftest(1_000_000, stream_handle()), "selftest")
    with pytest.raises(RuntimeError, match="bounded wait"):
        trainer.check_status()
    trainer.close()  # the status word was cleared by the failed check
