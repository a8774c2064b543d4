"""Sequence parallelism (time axis split over ranks, (W-1)-row halo exchange) on CPU
with gloo ranks.  A small differentiable torch restatement of the low-rank op
(reference.py:23-39) stands in for the CUDA kernels, so these tests check the
halo exchange itself: every rank's output and its x / z gradients must equal the
matching slice of the full-sequence computation, and the shared gradients (summed
over ranks) the full-sequence ones."""
from __future__ import annotations

import datetime
import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def ref_lowrank(x, z, U, static_w, residual=False):
    B, T, D = x.shape
    W = U.shape[-1] // D
    w = (z @ U).view(B, T, W, D)
    if static_w is not None:
        w = w + static_w
    y = sum(w[:, :, k] * F.pad(x, (0, 0, k, 0))[:, :T] for k in range(W))
    return y + x if residual else y


def ref_headwise(x, weight, static_w, residual=False):
    B, T, D = x.shape
    H, W = weight.shape[2], weight.shape[3]
    w = weight.repeat_interleave(D // H, dim=2)  # [B, T, D, W]
    if static_w is not None:
        w = w + static_w.t()
    y = sum(w[..., k] * F.pad(x, (0, 0, k, 0))[:, :T] for k in range(W))
    return y + x if residual else y


def _inputs(B=2, T=24, D=8, R=3, W=4, seed=0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(B, T, D, generator=g), torch.randn(B, T, R, generator=g),
            torch.randn(R, W * D, generator=g) * 0.5, torch.randn(W, D, generator=g) * 0.5,
            torch.randn(B, T, D, generator=g))


def _hw_inputs(B=2, T=24, D=8, H=4, W=4, seed=0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(B, T, D, generator=g), torch.randn(B, T, H, W, generator=g) * 0.5,
            torch.randn(W, D, generator=g) * 0.5, torch.randn(B, T, D, generator=g))


def _worker(rank, world, port, W, q, kind="lowrank"):
    try:
        from dynamic_conv1d_b200.sequence_parallel import sequence_parallel

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        if kind == "lowrank":
            x, z, U, sw, dy = _inputs(W=W)
            shared = [U, sw]
            fn = ref_lowrank
        else:
            x, z, sw, dy = _hw_inputs(W=W)
            shared = [sw]
            fn = ref_headwise
        T = x.shape[1]
        lo, hi = rank * T // world, (rank + 1) * T // world
        xl = x[:, lo:hi].clone().requires_grad_()
        zl = z[:, lo:hi].clone().requires_grad_()
        sh = [p.clone().requires_grad_() for p in shared]
        y = sequence_parallel(fn, xl, zl, *sh, residual=True, W=W)
        y.backward(dy[:, lo:hi])
        # the shared gradients come back already summed over the ranks
        q.put((rank, lo, hi, y.detach(), xl.grad, zl.grad) + tuple(p.grad for p in sh))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        import traceback

        q.put((rank, "error", traceback.format_exc()))


@pytest.mark.parametrize("world,W", [(2, 4), (3, 4), (3, 2), (2, 1)])
def test_sequence_parallel_matches_full_sequence(world, W):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, W, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for r in res:
        assert r[1] != "error", r[2]
    x, z, U, sw, dy = _inputs(W=W)
    leaves = [t.clone().requires_grad_() for t in (x, z, U, sw)]
    y = ref_lowrank(*leaves, residual=True)
    y.backward(dy)
    _check(res, leaves, y)


def _check(res, leaves, y):
    for rank, lo, hi, yl, gx, gz, *gshared in res:
        torch.testing.assert_close(yl, y.detach()[:, lo:hi], rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(gx, leaves[0].grad[:, lo:hi], rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(gz, leaves[1].grad[:, lo:hi], rtol=1e-5, atol=1e-5)
        for g, leaf in zip(gshared, leaves[2:]):
            torch.testing.assert_close(g, leaf.grad, rtol=1e-4, atol=1e-4)


def test_sequence_parallel_headwise_matches_full_sequence():
    world, W = 3, 4
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, W, q, "headwise")) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for r in res:
        assert r[1] != "error", r[2]
    x, w, sw, dy = _hw_inputs(W=W)
    leaves = [t.clone().requires_grad_() for t in (x, w, sw)]
    y = ref_headwise(*leaves, residual=True)
    y.backward(dy)
    _check(res, leaves, y)


def _short_worker(rank, world, port, q):
    try:
        from dynamic_conv1d_b200.sequence_parallel import sequence_parallel

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
        x, z, U, sw, _ = _inputs(T=12, W=4)
        # rank 1 holds only 2 steps (< W-1 = 3); rank 0 holds 10
        lo, hi = (0, 10) if rank == 0 else (10, 12)
        try:
            sequence_parallel(ref_lowrank, x[:, lo:hi], z[:, lo:hi], U, sw, residual=True, W=4)
            q.put((rank, "no error"))
        except ValueError as e:
            q.put((rank, "raised", str(e)))
        dist.destroy_process_group()
    except Exception:
        import traceback

        q.put((rank, "error", traceback.format_exc()))


def test_sequence_parallel_short_slice_raises_on_every_rank():
    """A slice shorter than W-1 on one rank makes every rank raise before the halo
    exchange (no rank is left waiting on a halo that is never sent)."""
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_short_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert [r[1] for r in res] == ["raised", "raised"], res
    assert "shortest slice holds 2" in res[0][2]
