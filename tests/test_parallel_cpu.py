"""Data-parallel host logic on CPU with two gloo ranks (no GPU).

The CUDA path shards the batch across ranks and all-reduces only the float32
shared-gradient accumulator (dU rows + the folded static_w row for lowrank,
dstatic_w for headwise).  These tests run that host logic -- ``shard_rows``,
``allreduce_shared_grad`` and the ``data_parallel`` context -- over real
``torch.distributed`` ranks, with the CPU oracle standing in for the kernels:
the reduced per-shard gradients must equal the full-batch gradients, and a rank
that leaves before the collective must make its peer fail with an error instead
of hanging."""
from __future__ import annotations

import datetime
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from dynamic_conv1d_b200.parallel import allreduce_shared_grad, current_group, data_parallel, shard_rows  # noqa: E402


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _inputs(B=5, T=37, D=16, R=3, W=3, H=4, seed=3):
    rng = np.random.default_rng(seed)
    f = lambda *s: rng.standard_normal(s).astype(np.float32)
    return dict(x=f(B, T, D), dy=f(B, T, D), z=f(B, T, R), U=f(R, W * D) * 0.5, sw=f(W, D) * 0.5,
                w=f(B, T, H, W), W=W, D=D)


def _dp_worker(rank, world, port, q):
    try:
        import oracle

        _init(rank, world, port)
        a = _inputs()
        shard = lambda k: shard_rows(torch.from_numpy(a[k]), rank, world).numpy()
        x, dy, z, w = shard("x"), shard("dy"), shard("z"), shard("w")
        # lowrank: the [R_kernel, W*D] fp32 accumulator = dU rows + the static row
        _, _, dU, dsw = oracle.lowrank_bwd(x, z, a["U"], a["sw"], dy, True)
        acc = torch.from_numpy(np.concatenate([dU, dsw.reshape(1, -1)], 0).astype(np.float32))
        with data_parallel() as g:
            assert current_group() is g
            allreduce_shared_grad(acc, current_group())
        assert current_group() is None
        # headwise: the [W, D] dstatic_w accumulator; dweight stays per shard
        _, dwt, hsw = oracle.headwise_bwd(x, w, a["sw"], dy, True)
        hacc = torch.from_numpy(hsw.astype(np.float32).copy())
        with data_parallel():
            allreduce_shared_grad(hacc, current_group())
        q.put((rank, acc.numpy(), hacc.numpy(), dwt, x.shape[0]))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, repr(e), None, None, None))


def test_shard_rows_partition():
    t = torch.arange(11)
    for world in (1, 2, 3, 4, 8):
        parts = [shard_rows(t, r, world) for r in range(world)]
        assert torch.equal(torch.cat(parts), t)
        sizes = [len(p) for p in parts]
        assert max(sizes) - min(sizes) <= 1


def test_data_parallel_needs_process_group():
    if dist.is_initialized():
        pytest.skip("a process group is already initialised in this process")
    with pytest.raises(RuntimeError):
        with data_parallel():
            pass
    assert current_group() is None
    buf = torch.ones(4)
    allreduce_shared_grad(buf, None)  # outside data_parallel: no-op
    assert torch.equal(buf, torch.ones(4))


def test_two_rank_allreduce_matches_full_batch():
    import oracle

    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_dp_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    results.sort(key=lambda r: r[0])
    for r in results:
        assert not isinstance(r[1], str), f"rank {r[0]} failed: {r[1]}"
    a = _inputs()
    _, _, dU, dsw = oracle.lowrank_bwd(a["x"], a["z"], a["U"], a["sw"], a["dy"], True)
    full = np.concatenate([dU, dsw.reshape(1, -1)], 0)
    _, dwt_full, hsw_full = oracle.headwise_bwd(a["x"], a["w"], a["sw"], a["dy"], True)
    for rank, acc, hacc, dwt, rows in results:
        np.testing.assert_allclose(acc, full, rtol=1e-5, atol=1e-4)
        np.testing.assert_allclose(hacc, hsw_full, rtol=1e-5, atol=1e-4)
    # dweight is not reduced: the shards concatenate to the full-batch dweight
    np.testing.assert_allclose(np.concatenate([r[3] for r in results], 0), dwt_full, rtol=1e-5, atol=1e-5)
    assert [r[4] for r in results] == [3, 2]


def _leaver_worker(rank, world, port, q):
    try:
        _init(rank, world, port, timeout_s=5)
        if rank == 1:
            q.put((rank, "left"))
            return  # leaves between steps, before the collective, without destroying the group
        buf = torch.ones(8)
        try:
            with data_parallel():
                allreduce_shared_grad(buf, current_group())
            q.put((rank, "no error"))
        except Exception as e:  # the expected outcome: the collective ends with an error
            q.put((rank, "error:" + type(e).__name__))
    except Exception as e:
        q.put((rank, "setup failed: " + repr(e)))


def test_rank_that_leaves_makes_peer_fail_not_hang():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_leaver_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=180) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert out[1] == "left"
    assert out[0].startswith("error:"), out[0]
