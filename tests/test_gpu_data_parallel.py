"""The data-parallel backward path on a GPU, over a one-rank NCCL process group.

Inside ``data_parallel()`` the backward of both ops takes the other branch: the
kernels leave the float32 shared-gradient accumulator unconverted, it is
all-reduced through torch.distributed (NCCL), and then cast to the parameter
dtype (lowrank: one cast of the whole [R_kernel, W*D] buffer, returned as row
views).  A SUM over one rank is the identity, so every gradient must equal the
single-process path bit for bit.  Runs in a child process so the process group
never leaks into other tests."""
from __future__ import annotations

import os
import socket
import subprocess
import sys
import textwrap

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = textwrap.dedent(
    """
    import sys, datetime
    import torch, torch.distributed as dist
    sys.path.insert(0, {root!r})
    from dynamic_conv1d_b200 import (data_parallel, headwise_dynamic_convolution, lowrank_dynamic_convolution,
                                     lowrank_dynamic_convolution_grouped)
    dist.init_process_group("nccl", init_method="tcp://127.0.0.1:{port}", rank=0, world_size=1,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", 0))
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(5)
    bf = torch.bfloat16
    def rnd(*s, scale=1.0):
        return (torch.randn(*s, generator=g) * scale).to(bf).to(dev)

    def grads(fn, cpu_leaves, dy, dp):
        leaves = [t.clone().requires_grad_() for t in cpu_leaves]
        if dp:
            with data_parallel():
                y = fn(*leaves, residual=True)
                y.backward(dy)
        else:
            y = fn(*leaves, residual=True)
            y.backward(dy)
        torch.cuda.synchronize()
        return [y.detach()] + [l.grad for l in leaves]

    B, T, D, W = 2, 200, 256, 4
    x, dy = rnd(B, T, D), rnd(B, T, D)
    cases = {{
        "lowrank_static": (lowrank_dynamic_convolution, [x, rnd(B, T, 15), rnd(15, W * D, scale=0.25), rnd(W, D, scale=0.3)]),
        "lowrank_nostatic": (lowrank_dynamic_convolution, [x, rnd(B, T, 16), rnd(16, W * D, scale=0.25)]),
        "headwise_hs32": (headwise_dynamic_convolution, [x, rnd(B, T, D // 32, W, scale=0.3), rnd(W, D, scale=0.3)]),
        "lowrank_grouped": (lowrank_dynamic_convolution_grouped,
                            [rnd(B, T, 3 * D), rnd(B, T, 3 * 15), rnd(3, 15, W * D, scale=0.25), rnd(3, W, D, scale=0.3)]),
    }}
    dy3 = rnd(B, T, 3 * D)
    for name, (fn, leaves) in cases.items():
        d = dy3 if name == "lowrank_grouped" else dy
        ref = grads(fn, leaves, d, dp=False)
        got = grads(fn, leaves, d, dp=True)
        for i, (a, b) in enumerate(zip(ref, got)):
            assert a.shape == b.shape and a.dtype == b.dtype, (name, i, a.shape, b.shape, a.dtype, b.dtype)
            assert torch.equal(a, b), (name, i, (a.float() - b.float()).abs().max().item())
        print("ok", name)
    dist.destroy_process_group()
    """
)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_data_parallel_backward_matches_single_process(cuda_device):
    code = CHILD.format(root=ROOT, port=_free_port())
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=240)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert r.stdout.count("ok ") == 4, r.stdout


THREAD_CHILD = textwrap.dedent(
    """
    import sys, threading
    import torch
    sys.path.insert(0, {root!r})
    from dynamic_conv1d_b200 import _lib
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(9)
    B, T, D, R, W = 2, 130, 256, 15, 4
    bf = torch.bfloat16
    x = torch.randn(B, T, D, generator=g).to(bf).to(dev)
    z = torch.randn(B, T, R, generator=g).to(bf).to(dev)
    U = (torch.randn(R, W * D, generator=g) * 0.25).to(bf).to(dev)
    sw = (torch.randn(W, D, generator=g) * 0.3).to(bf).to(dev)
    nb = lib.dynconv_lr_fwd_workspace_bytes(B, T, D, R, W, 0, 1)
    ws = torch.empty(nb, dtype=torch.uint8, device=dev)
    torch.cuda.synchronize()

    def call(y):
        # a thread that has made no CUDA runtime call of its own
        st = _lib.stream_of(x)
        status[0] = lib.dynconv_lr_fwd(_lib.ptr(x), _lib.ptr(z), _lib.ptr(U), _lib.ptr(sw), _lib.ptr(y), _lib.ptr(ws),
                                       nb, B, T, D, R, W, 0, 1, st)
        if status[0] != 0:
            status.append(lib.dynconv_last_error().decode())

    y_thread, y_main = torch.empty_like(x), torch.empty_like(x)
    status = [None]
    th = threading.Thread(target=call, args=(y_thread,))
    th.start(); th.join()
    assert status[0] == 0, status
    call(y_main)
    assert status[0] == 0, status
    torch.cuda.synchronize()
    assert torch.equal(y_thread, y_main)
    print("ok thread")
    """
)


def test_entry_point_from_a_fresh_thread(cuda_device):
    """TMA descriptor encoding is a driver call that needs a current context; the
    library binds the device's primary context itself on a thread that has none."""
    r = subprocess.run([sys.executable, "-c", THREAD_CHILD.format(root=ROOT)], capture_output=True, text=True,
                       timeout=240)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "ok thread" in r.stdout, r.stdout


SP_CHILD = textwrap.dedent(
    """
    import sys, datetime
    import numpy as np
    import torch, torch.distributed as dist
    sys.path.insert(0, {root!r})
    import oracle
    from dynamic_conv1d_b200 import headwise_dynamic_convolution_sp, lowrank_dynamic_convolution_sp
    dist.init_process_group("nccl", init_method="tcp://127.0.0.1:{port}", rank=0, world_size=1,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", 0))
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(6)
    bf = torch.bfloat16
    def rnd(*s, scale=1.0):
        return (torch.randn(*s, generator=g) * scale).to(bf)
    def rel(a, ref):
        a = a.detach().float().cpu().numpy().astype(np.float64)
        return np.linalg.norm(a - ref) / max(np.linalg.norm(ref), 1e-30)
    B, T, D, W = 2, 200, 256, 4
    x, dy = rnd(B, T, D), rnd(B, T, D)
    cases = {{
        "lowrank": (lowrank_dynamic_convolution_sp, oracle.lowrank_fwd, oracle.lowrank_bwd,
                    [x, rnd(B, T, 15), rnd(15, W * D, scale=0.25), rnd(W, D, scale=0.3)]),
        "headwise": (headwise_dynamic_convolution_sp, oracle.headwise_fwd, oracle.headwise_bwd,
                     [x, rnd(B, T, D // 32, W, scale=0.3), rnd(W, D, scale=0.3)]),
    }}
    f = lambda t: t.float().numpy()
    for name, (fn_sp, ofwd, obwd, cpu) in cases.items():
        leaves = [t.to(dev).requires_grad_() for t in cpu]
        y = fn_sp(*leaves, residual=True)
        y.backward(dy.to(dev))
        torch.cuda.synchronize()
        refs = [ofwd(*map(f, cpu), True)] + list(obwd(*map(f, cpu), f(dy), True))
        for i, (a, ref) in enumerate(zip([y] + [l.grad for l in leaves], refs)):
            e = rel(a, ref)
            assert e <= (1e-2 if i == 0 else 2e-2), (name, i, e)
        print("ok", name)
    dist.destroy_process_group()
    """
)


def test_sequence_parallel_one_rank_matches_oracle(cuda_device):
    """Time-sharded wrappers on one NCCL rank: the halo is the zero padding; output
    and all gradients match the CPU oracle (rel-L2 1e-2 for y, 2e-2 for gradients)."""
    code = SP_CHILD.format(root=ROOT, port=_free_port())
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=240)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert r.stdout.count("ok ") == 2, r.stdout


def test_tensors_on_a_non_current_device():
    """Tensors on cuda:1 while cuda:0 is current: the Functions make the tensors'
    device current around their library calls (needs two GPUs)."""
    import torch

    from dynamic_conv1d_b200 import headwise_dynamic_convolution, lowrank_dynamic_convolution

    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    dev = torch.device("cuda", 1)
    g = torch.Generator().manual_seed(8)
    bf = torch.bfloat16

    def rnd(*s, scale=1.0):
        return (torch.randn(*s, generator=g) * scale).to(bf)

    B, T, D, W = 2, 150, 256, 4
    cpu = {"x": rnd(B, T, D), "dy": rnd(B, T, D), "z": rnd(B, T, 15), "U": rnd(15, W * D, scale=0.25),
           "sw": rnd(W, D, scale=0.3), "w": rnd(B, T, D // 32, W, scale=0.3)}

    def run(current):
        torch.cuda.set_device(current)
        t = {k: v.to(dev) for k, v in cpu.items()}
        outs = []
        for fn, args in ((lowrank_dynamic_convolution, ["x", "z", "U", "sw"]),
                         (headwise_dynamic_convolution, ["x", "w", "sw"])):
            leaves = [t[a].clone().requires_grad_() for a in args]
            y = fn(*leaves, residual=True)
            y.backward(t["dy"])
            torch.cuda.synchronize(dev)
            outs += [y.detach()] + [l.grad for l in leaves]
        return outs

    other = run(0)
    same = run(1)
    torch.cuda.set_device(0)
    for a, b in zip(other, same):
        assert a.device == dev and torch.equal(a, b)


SP2_SCRIPT = textwrap.dedent(
    """
    import datetime, os, sys
    import numpy as np
    import torch, torch.distributed as dist
    sys.path.insert(0, {root!r})
    import oracle
    from dynamic_conv1d_b200 import headwise_dynamic_convolution_sp, lowrank_dynamic_convolution_sp
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    g = torch.Generator().manual_seed(12)
    bf = torch.bfloat16
    def rnd(*s, scale=1.0):
        return (torch.randn(*s, generator=g) * scale).to(bf)
    def rel(a, ref):
        a = a.detach().float().cpu().numpy().astype(np.float64)
        return np.linalg.norm(a - ref) / max(np.linalg.norm(ref), 1e-30)
    B, T, D, W = 2, 300, 256, 4
    x, dy = rnd(B, T, D), rnd(B, T, D)
    cases = {{
        "lowrank": (lowrank_dynamic_convolution_sp, oracle.lowrank_fwd, oracle.lowrank_bwd,
                    [x, rnd(B, T, 15), rnd(15, W * D, scale=0.25), rnd(W, D, scale=0.3)], 2),
        "headwise": (headwise_dynamic_convolution_sp, oracle.headwise_fwd, oracle.headwise_bwd,
                     [x, rnd(B, T, D // 32, W, scale=0.3), rnd(W, D, scale=0.3)], 2),
    }}
    lo, hi = rank * T // world, (rank + 1) * T // world
    f = lambda t: t.float().numpy()
    for name, (fn_sp, ofwd, obwd, cpu, n_local) in cases.items():
        # time-sharded: x and the mixing input are split, the shared parameters replicated
        leaves = [t[:, lo:hi].contiguous().to(dev) if i < n_local else t.to(dev) for i, t in enumerate(cpu)]
        leaves = [t.requires_grad_() for t in leaves]
        y = fn_sp(*leaves, residual=True)
        y.backward(dy[:, lo:hi].contiguous().to(dev))
        torch.cuda.synchronize()
        # the full sequence on the CPU oracle; this rank's slice of it
        ry = ofwd(*map(f, cpu), True)
        rg = obwd(*map(f, cpu), f(dy), True)
        refs = [ry[:, lo:hi]] + [r[:, lo:hi] for r in rg[:n_local]] + list(rg[n_local:])
        for i, (a, ref) in enumerate(zip([y] + [l.grad for l in leaves], refs)):
            e = rel(a, ref)
            assert e <= (1e-2 if i == 0 else 2e-2), (name, rank, i, e)
        print("ok", name, rank, flush=True)
    dist.barrier()
    dist.destroy_process_group()
    """
)


def test_sequence_parallel_two_gpus(tmp_path):
    """Time axis split over two GPUs (NCCL point-to-point halo exchange, shared
    gradients all-reduced): each rank's output and gradients match its slice of the
    full-sequence CPU oracle (needs two GPUs)."""
    import torch

    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    script = tmp_path / "sp2.py"
    script.write_text(SP2_SCRIPT.format(root=ROOT))
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                        "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), str(script)],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert r.stdout.count("ok ") == 4, r.stdout


DP2_SCRIPT = textwrap.dedent(
    """
    import datetime, os, sys
    import numpy as np
    import torch, torch.distributed as dist
    sys.path.insert(0, {root!r})
    import oracle
    from dynamic_conv1d_b200 import data_parallel, lowrank_dynamic_convolution, lowrank_dynamic_convolution_grouped
    from dynamic_conv1d_b200 import parallel
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    g = torch.Generator().manual_seed(21)
    bf = torch.bfloat16
    def rnd(*s, scale=1.0):
        return (torch.randn(*s, generator=g) * scale).to(bf)
    def rel(a, ref):
        a = a.detach().float().cpu().numpy().astype(np.float64)
        return np.linalg.norm(a - ref) / max(np.linalg.norm(ref), 1e-30)
    f = lambda t: t.float().numpy()
    B, T, D, R, W = 2 * world, 300, 256, 15, 4
    x, dy, z = rnd(B, T, D), rnd(B, T, D), rnd(B, T, R, scale=0.5)
    U, sw = rnd(R, W * D, scale=0.25), rnd(W, D, scale=0.3)
    rows = slice(2 * rank, 2 * rank + 2)
    ry = oracle.lowrank_fwd(f(x), f(z), f(U), f(sw), True)
    rdx, rdz, rdU, rdsw = oracle.lowrank_bwd(f(x), f(z), f(U), f(sw), f(dy), True)

    # eager, three calls (both landing parities, then the first again)
    for it in range(3):
        leaves = [x[rows].to(dev).requires_grad_(), z[rows].to(dev).requires_grad_(),
                  U.to(dev).requires_grad_(), sw.to(dev).requires_grad_()]
        with data_parallel():
            y = lowrank_dynamic_convolution(*leaves, residual=True)
            y.backward(dy[rows].to(dev))
        torch.cuda.synchronize()
        assert parallel._comms, "the fused data-parallel path was not used"
        errs = [rel(y, ry[rows]), rel(leaves[0].grad, rdx[rows]), rel(leaves[1].grad, rdz[rows]),
                rel(leaves[2].grad, rdU), rel(leaves[3].grad, rdsw)]
        assert errs[0] <= 1e-2 and max(errs[1:]) <= 2e-2, (it, errs)
        # every rank holds the same shared gradients, bit for bit
        for t in (leaves[2].grad, leaves[3].grad):
            allg = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(allg, t.contiguous())
            assert all(torch.equal(allg[0], a) for a in allg), it
    print("ok eager", rank, flush=True)

    # grouped (Q/K/V) op: one stacked reduction
    G = 3
    xg, dyg, zg = rnd(B, T, G * D), rnd(B, T, G * D), rnd(B, T, G * R, scale=0.5)
    Ug, swg = rnd(G, R, W * D, scale=0.25), rnd(G, W, D, scale=0.3)
    leaves = [xg[rows].to(dev).requires_grad_(), zg[rows].to(dev).requires_grad_(),
              Ug.to(dev).requires_grad_(), swg.to(dev).requires_grad_()]
    with data_parallel():
        y = lowrank_dynamic_convolution_grouped(*leaves, residual=True)
        y.backward(dyg[rows].to(dev))
    torch.cuda.synchronize()
    for gi in range(G):
        sl, slr = slice(gi * D, (gi + 1) * D), slice(gi * R, (gi + 1) * R)
        _, _, gU, gsw = oracle.lowrank_bwd(f(xg)[..., sl], f(zg)[..., slr], f(Ug[gi]), f(swg[gi]), f(dyg)[..., sl], True)
        assert rel(leaves[2].grad[gi], gU) <= 2e-2 and rel(leaves[3].grad[gi], gsw) <= 2e-2, gi
    print("ok grouped", rank, flush=True)

    # the step captured in a CUDA graph and replayed: the call counter lives on the device
    leaves = [x[rows].to(dev).requires_grad_(), z[rows].to(dev).requires_grad_(),
              U.to(dev).requires_grad_(), sw.to(dev).requires_grad_()]
    dyd = dy[rows].to(dev)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s), data_parallel():
        for _ in range(2):
            for l in leaves:
                l.grad = None
            lowrank_dynamic_convolution(*leaves, residual=True).backward(dyd)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    for l in leaves:
        l.grad = None
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph), data_parallel():
        lowrank_dynamic_convolution(*leaves, residual=True).backward(dyd)
    for it in range(4):
        graph.replay()
        torch.cuda.synchronize()
        assert rel(leaves[2].grad, rdU) <= 2e-2 and rel(leaves[3].grad, rdsw) <= 2e-2, it
    from dynamic_conv1d_b200 import _lib
    _lib.check_device(leaves[0])
    del graph
    print("ok graph", rank, flush=True)
    dist.barrier()
    dist.destroy_process_group()
    """
)


def test_fused_data_parallel_two_gpus(tmp_path):
    """The lowrank backward with the shared-gradient sum done inside the kernel over
    peer memory (two GPUs): gradients match the full-batch oracle, are bit-identical
    on both ranks, and stay right over repeated calls and CUDA-graph replays."""
    import torch

    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    script = tmp_path / "dp2.py"
    script.write_text(DP2_SCRIPT.format(root=ROOT))
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                        "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), str(script)],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    for tag in ("ok eager", "ok grouped", "ok graph"):
        assert r.stdout.count(tag) == 2, r.stdout
