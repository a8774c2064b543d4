"""Benchmark of the dynamic short convolution hot path on B200 (driver contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (N > 1, one rank per GPU)

One step = forward + backward of ``lowrank_dynamic_convolution`` (the metric of
"fwd+bwd Mtokens/s and % of HBM roofline, lowrank R=16 D=2048
W=4") on the workload of configs[3]: B=4, T=4096, D=2048, W=4, z [B,T,15],
U [15, 8192] ~ N(0, 1/15), static_w ~ U(-0.5, 0.5) fused as the 16th rank,
residual=True, bf16, upstream gradient dy ~ N(0,1) (seeded synthetic data).
With N GPUs every rank runs that per-GPU workload on its own batch shard
(weak scaling, global batch 4N) and the float32 dU/dstatic_w accumulator is
all-reduced over NCCL inside the backward.

Reported (one JSON line on rank 0):
  value       Mtokens/s of the whole job, device-timed with CUDA events per step
              (max over ranks), inputs resident in HBM, L2 flushed between steps
              (a 256 MiB write outside the timed events), the fwd+bwd step
              replayed from a CUDA graph so host overhead is not measured;
  e2e         the same metric through the public autograd API with the step's
              inputs (x, z, dy) copied from pinned host memory and all results
              (y, dx, dz, dU, dstatic_w) copied back, inside the timed region
              (pipelined over batch rows so uploads and downloads overlap);
  roofline    the dominant kernel (the lowrank backward call) -- algorithmic bytes
              per launch / its CUDA-event duration, against MEASURED_PEAKS.json;
  cpu_baseline the numpy oracle (a restatement of the reference's reference.py) on
              the host cores, on a bounded sample of the same workload.

``--impl reference`` times the reference's CPU implementation of the path (the
oracle port) on the host cores with the same workload/metric; rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "fwd+bwd Mtokens/s and % of HBM roofline, lowrank R=16 D=2048 W=4"
UNIT = "Mtokens/s"

WORKLOADS = {
    # BASELINE.json configs[3] (the metric's config) -- per GPU
    "lowrank": dict(kind="lowrank", B=4, T=4096, D=2048, R=15, W=4, static=True, residual=True),
    # configs[4] per-GPU shard (B=64 over 8 GPUs)
    "lowrank_dp": dict(kind="lowrank", B=8, T=8192, D=4096, R=31, W=4, static=True, residual=True),
    # configs[1], configs[2]
    "headwise_hs32": dict(kind="headwise", B=4, T=4096, D=2048, H=64, W=4, static=True, residual=True),
    "headwise_hs1": dict(kind="headwise", B=4, T=4096, D=2048, H=2048, W=4, static=True, residual=True),
    # shapes the reference accepts outside the tensor-core envelope (not BASELINE configs; run only
    # with --workload): the cfg4 workload with W = 8 taps, and with rank 63 + static (R_kernel = 64)
    "lowrank_w8": dict(kind="lowrank", B=4, T=4096, D=2048, R=15, W=8, static=True, residual=True),
    "lowrank_r63": dict(kind="lowrank", B=4, T=4096, D=2048, R=63, W=4, static=True, residual=True),
}


def algorithmic_bytes(wl: dict, e: int = 2) -> tuple[int, int]:
    """(forward, backward) bytes that must cross HBM once: every tensor read or written once."""
    B, T, D, W = wl["B"], wl["T"], wl["D"], wl["W"]
    N = B * T
    sw = W * D if wl["static"] else 0
    if wl["kind"] == "lowrank":
        R = wl["R"]
        fwd = e * (2 * N * D + N * R + R * W * D + sw)
        bwd = e * (3 * N * D + 2 * N * R + 2 * R * W * D + 2 * sw)
    else:
        H = wl["H"]
        fwd = e * (2 * N * D + N * H * W + sw)
        bwd = e * (3 * N * D + 2 * N * H * W + 2 * sw)
    return fwd, bwd


# ----------------------------------------------------------------- inputs

def make_inputs_np(wl: dict, rows: int | None = None, T: int | None = None, seed: int = 0):
    """Seeded synthetic inputs (float32 arrays holding bf16-representable values)."""
    import torch

    B = rows if rows is not None else wl["B"]
    TT = T if T is not None else wl["T"]
    D, W = wl["D"], wl["W"]
    g = torch.Generator().manual_seed(seed)

    def bf(t):
        return t.to(torch.bfloat16).float().numpy()

    out = {"x": bf(torch.randn(B, TT, D, generator=g)), "dy": bf(torch.randn(B, TT, D, generator=g))}
    if wl["kind"] == "lowrank":
        R = wl["R"]
        out["z"] = bf(torch.randn(B, TT, R, generator=g))
        out["U"] = bf(torch.randn(R, W * D, generator=g) / np.sqrt(R))
    else:
        out["weight"] = bf(torch.randn(B, TT, wl["H"], W, generator=g))
    out["static_w"] = bf(torch.rand(W, D, generator=g) - 0.5) if wl["kind"] == "lowrank" else bf(torch.randn(W, D, generator=g))
    return out


# ----------------------------------------------------------------- CPU leg

def usable_cores() -> int:
    """Host cores this process may run on (the affinity mask), at least 1."""
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except (AttributeError, OSError):
        return max(1, os.cpu_count() or 1)


def cpu_oracle_step(wl: dict, a: dict, threads: int):
    """fwd+bwd of the oracle on the sample `a`, one batch row per task, `threads`
    workers.  numpy releases the GIL inside its array kernels and BLAS is held to
    one thread per worker, so the rows run in parallel on `threads` cores."""
    import oracle  # test infrastructure; only the cpu_baseline / reference legs use it
    from concurrent.futures import ThreadPoolExecutor

    from threadpoolctl import threadpool_limits

    B = a["x"].shape[0]
    res = bool(wl["residual"])

    def one(b):
        sl = slice(b, b + 1)
        if wl["kind"] == "lowrank":
            y = oracle.lowrank_fwd(a["x"][sl], a["z"][sl], a["U"], a["static_w"], res)
            g = oracle.lowrank_bwd(a["x"][sl], a["z"][sl], a["U"], a["static_w"], a["dy"][sl], res)
        else:
            y = oracle.headwise_fwd(a["x"][sl], a["weight"][sl], a["static_w"], res)
            g = oracle.headwise_bwd(a["x"][sl], a["weight"][sl], a["static_w"], a["dy"][sl], res)
        return y, g

    with threadpool_limits(limits=1), ThreadPoolExecutor(max_workers=threads) as ex:
        outs = list(ex.map(one, range(B)))
    # shared gradients are summed over rows, as the full-batch reference does
    acc = outs[0][1][2].copy()
    for o in outs[1:]:
        acc += o[1][2]
    return acc


def cpu_sample(wl: dict, cores: int, Ts: int, seed: int = 1) -> dict:
    """The bounded CPU sample: one independent segment of Ts steps per core (the op is
    local in time, so the work per token does not depend on the segment length)."""
    return make_inputs_np(wl, rows=cores, T=min(wl["T"], Ts), seed=seed)


def cpu_baseline(wl: dict, steps: int = 3, budget_s: float = 20.0) -> dict:
    """Time the oracle on a bounded sample spread over every usable host core."""
    cores = usable_cores()
    Ts = 512
    a = cpu_sample(wl, cores, Ts)
    t0 = time.perf_counter()
    cpu_oracle_step(wl, a, cores)
    first = time.perf_counter() - t0
    n = max(1, min(steps, int(budget_s / max(first, 1e-3))))
    best = first
    for _ in range(n):
        t0 = time.perf_counter()
        cpu_oracle_step(wl, a, cores)
        best = min(best, time.perf_counter() - t0)
    toks = a["x"].shape[0] * a["x"].shape[1]
    return {
        "value": toks / best / 1e6,
        "unit": UNIT,
        "cores": cores,
        "host_cpus": os.cpu_count(),
        "kind": "port",
        "sample": f"{cores} segments x {a['x'].shape[1]} steps (one per core, D={wl['D']}), numpy restatement of "
                  f"reference.py fwd+bwd, best of {n + 1}",
    }


def run_reference_arm(args, wl: dict) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cores = usable_cores()
    Ts = 512
    a = cpu_sample(wl, cores, Ts)
    for _ in range(args.warmup):
        cpu_oracle_step(wl, a, cores)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        cpu_oracle_step(wl, a, cores)
        times.append(time.perf_counter() - t0)
    tot = sum(times)
    rows, Tsamp = a["x"].shape[0], a["x"].shape[1]
    toks = rows * Tsamp * args.steps
    val = toks / tot / 1e6
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": val,
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": tot / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": args.workload, **wl, "sample_segments": rows, "sample_T": Tsamp},
        "cpu_baseline": {
            "value": val,
            "unit": UNIT,
            "cores": cores,
            "host_cpus": os.cpu_count(),
            "kind": "port",
            "sample": f"{rows} segments x {Tsamp} steps per step (one per core); numpy restatement of "
                      "reference.py fwd+bwd",
        },
        "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while active."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def wait_first_sample(self, timeout: float = 5.0):
        t_end = time.time() + timeout
        while self.proc is not None and not self.lines and time.time() < t_end:
            time.sleep(0.02)
        self._mark = len(self.lines)

    def mark(self):
        pass

    def samples_since_mark(self) -> int:
        return len(self.lines) - getattr(self, "_mark", 0) if self.proc is not None else 99

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines[getattr(self, "_mark", 0):]:
            p = [s.strip() for s in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx = float(p[2])
            except ValueError:
                continue
            for nm, v in zip(names, p[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": mx,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }


# ----------------------------------------------------------------- GPU leg

def _peaks() -> tuple[float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def _traffic_from_profiles(workload: str):
    p = os.path.join(ROOT, "profiles", "roofline_traffic.json")
    try:
        with open(p) as f:
            return json.load(f).get(workload)
    except Exception:
        return None


def device_inputs(wl: dict, dev, seed: int):
    """Seeded synthetic inputs generated on the device (bf16), with BASELINE's
    distributions; the shared parameters (U, static_w) use one seed on every rank."""
    import torch

    B, T, D, W = wl["B"], wl["T"], wl["D"], wl["W"]
    bf = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(seed)
    gs = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn(B, T, D, device=dev, generator=g).to(bf).requires_grad_()
    dy = torch.randn(B, T, D, device=dev, generator=g).to(bf)
    if wl["kind"] == "lowrank":
        R = wl["R"]
        z = torch.randn(B, T, R, device=dev, generator=g).to(bf).requires_grad_()
        U = (torch.randn(R, W * D, device=dev, generator=gs) / np.sqrt(R)).to(bf).requires_grad_()
        sw = (torch.rand(W, D, device=dev, generator=gs) - 0.5).to(bf).requires_grad_()
        return [x, z, U, sw], dy
    wgt = torch.randn(B, T, wl["H"], W, device=dev, generator=g).to(bf).requires_grad_()
    sw = torch.randn(W, D, device=dev, generator=gs).to(bf).requires_grad_()
    return [x, wgt, sw], dy


def _backward(y, dy):
    """y.backward(dy), or one backward over several outputs (a tuple of y and of dy)."""
    import torch

    if isinstance(y, (tuple, list)):
        torch.autograd.backward(list(y), list(dy))
    else:
        y.backward(dy)


class DeviceStep:
    """One fwd+bwd step of `fn` on resident inputs, captured in a CUDA graph (eager if
    capture fails), timed with CUDA events per step with an L2 flush before each."""

    def __init__(self, args, wl, leaves, dy, fn, dev, world, dp_ctx, flush):
        import torch

        self.args, self.wl, self.leaves, self.dy, self.fn = args, wl, leaves, dy, fn
        self.dev, self.world, self.dp_ctx, self.flush = dev, world, dp_ctx, flush
        self.res = bool(wl["residual"])
        self.graph = None
        self.graph_error = None
        with dp_ctx():
            for _ in range(max(args.warmup, 3)):
                self.step()
        torch.cuda.synchronize()
        if not args.no_graph:
            try:
                s = torch.cuda.Stream(device=dev)
                s.wait_stream(torch.cuda.current_stream(dev))
                with torch.cuda.stream(s), dp_ctx():
                    for _ in range(2):
                        self.step()
                torch.cuda.current_stream(dev).wait_stream(s)
                torch.cuda.synchronize()
                graph = torch.cuda.CUDAGraph()
                for l in leaves:
                    l.grad = None
                with torch.cuda.graph(graph), dp_ctx():
                    _backward(fn(*leaves, residual=self.res), dy)
                torch.cuda.synchronize()
                self.graph = graph
            except Exception as e:  # pragma: no cover - reported in the JSON line
                self.graph_error = repr(e)[:200]

    def step(self):
        for l in self.leaves:
            l.grad = None
        y = self.fn(*self.leaves, residual=self.res)
        _backward(y, self.dy)
        return y

    def run_one(self):
        if self.graph is not None:
            self.graph.replay()
        else:
            with self.dp_ctx():
                self.step()

    def measure(self, steps: int, local: int) -> dict:
        """K timed steps (after W untimed), max over ranks; clocks sampled meanwhile."""
        import torch
        import torch.distributed as dist

        from dynamic_conv1d_b200 import _lib

        lib = _lib.load()
        world, dev = self.world, self.dev
        for _ in range(self.args.warmup):
            self.run_one()
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        launches0 = lib.dynconv_launch_count()
        with ClockSampler(local) as clk:
            clk.wait_first_sample()
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            wall0 = time.perf_counter()
            for i in range(steps):
                self.flush.zero_()
                starts[i].record()
                self.run_one()
                ends[i].record()
            torch.cuda.synchronize()
            wall = time.perf_counter() - wall0
            launches = lib.dynconv_launch_count() - launches0
            _lib.check_device(self.leaves[0])  # raises if a kernel gave up a bounded wait
            # The timed region is a few milliseconds, shorter than the 200 ms sampling
            # period: keep the same step running (untimed) until the sampler has seen
            # at least 3 samples under this load.  Every replay holds the data-parallel
            # all-reduce, so all ranks must run the same number of them: each round the
            # ranks agree (MAX) on whether any of them still needs samples.
            clk.mark()
            t_end = time.perf_counter() + 5.0
            while True:
                need = clk.samples_since_mark() < 3 and time.perf_counter() < t_end
                if world > 1:
                    flag = torch.tensor([1 if need else 0], device=dev, dtype=torch.int32)
                    dist.all_reduce(flag, op=dist.ReduceOp.MAX)
                    need = bool(flag.item())
                if not need:
                    break
                for _ in range(20):
                    self.flush.zero_()
                    self.run_one()
                torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        total_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
        t = torch.tensor([total_ms], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
        # graph replays launch without going through the library: count one step eagerly
        if self.graph is not None:
            l0 = lib.dynconv_launch_count()
            with self.dp_ctx():
                self.step()
            torch.cuda.synchronize()
            launches = (lib.dynconv_launch_count() - l0) * steps
        return {"total_ms": total_ms, "wall": wall, "launches": launches, "clocks": clk.summary()}

    def release(self):
        self.graph = None


def _dp_ctx_factory(world):
    import contextlib

    from dynamic_conv1d_b200 import data_parallel

    def dp_ctx():
        return data_parallel() if world > 1 else contextlib.nullcontext()

    return dp_ctx


def sub_workload(args, name: str, wl: dict, dev, world: int, local: int, rank: int, flush, scaling: str) -> dict:
    """The same device-timed measurement on another BASELINE config (no e2e / CPU leg):
    value, step roofline fraction, the backward kernel's roofline and the clocks."""
    import torch

    from dynamic_conv1d_b200 import headwise_dynamic_convolution, lowrank_dynamic_convolution

    fn = lowrank_dynamic_convolution if wl["kind"] == "lowrank" else headwise_dynamic_convolution
    leaves, dy = device_inputs(wl, dev, seed=100 + rank)
    ds = DeviceStep(args, wl, leaves, dy, fn, dev, world, _dp_ctx_factory(world), flush)
    steps = max(5, min(args.steps, 10))
    m = ds.measure(steps, local)
    roof = kernel_roofline(args, wl, leaves, dy, fn, flush, dev, workload=name)
    ds.release()
    fwd_b, bwd_b = algorithmic_bytes(wl)
    peak = _peaks()[0]
    ms = m["total_ms"] / steps
    out = {
        "value": world * wl["B"] * wl["T"] * steps / (m["total_ms"] / 1e3) / 1e6,
        "unit": UNIT,
        "ms_per_step": ms,
        "steps": steps,
        "scaling": scaling,
        "config": {**wl, "global_batch": wl["B"] * world, "parallelism": f"dp{world}"},
        "hbm_roofline_frac_step": (fwd_b + bwd_b) / (ms / 1e3) / (peak * 1e9),
        "roofline": roof,
        "clocks": m["clocks"],
        "gpu_launches": m["launches"],
    }
    del leaves, dy, ds
    torch.cuda.empty_cache()
    return out


def qkv_workload(args, dev, world: int, local: int, rank: int, flush) -> dict:
    """The query, key and value convolutions of one attention layer on configs[3]'s
    shapes (README.md:86-105: three LowRankDynamicShortConvolution modules): the
    grouped op -- one forward and one backward launch over the fused [B, T, 3D]
    activations, one stacked dU all-reduce under DP -- against three separate
    calls on already-contiguous per-group tensors, both device-timed the same way."""
    import torch

    from dynamic_conv1d_b200 import lowrank_dynamic_convolution, lowrank_dynamic_convolution_grouped

    wl = dict(WORKLOADS["lowrank"])
    G, B, T, D, R, W = 3, wl["B"], wl["T"], wl["D"], wl["R"], wl["W"]
    bf = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(300 + rank)
    gs = torch.Generator(device=dev).manual_seed(9)
    x = torch.randn(B, T, G * D, device=dev, generator=g).to(bf)
    dy = torch.randn(B, T, G * D, device=dev, generator=g).to(bf)
    z = torch.randn(B, T, G * R, device=dev, generator=g).to(bf)
    U = (torch.randn(G, R, W * D, device=dev, generator=gs) / np.sqrt(R)).to(bf)
    sw = (torch.rand(G, W, D, device=dev, generator=gs) - 0.5).to(bf)
    leaves = [t.clone().requires_grad_() for t in (x, z, U, sw)]
    dp_ctx = _dp_ctx_factory(world)
    steps = max(5, min(args.steps, 10))
    ds = DeviceStep(args, wl, leaves, dy, lowrank_dynamic_convolution_grouped, dev, world, dp_ctx, flush)
    m = ds.measure(steps, local)
    ds.release()

    sep = []
    for i in range(G):
        sep += [x[..., i * D:(i + 1) * D].contiguous(), z[..., i * R:(i + 1) * R].contiguous(), U[i].contiguous(),
                sw[i].contiguous()]
    sep = [t.requires_grad_() for t in sep]
    dy3 = tuple(dy[..., i * D:(i + 1) * D].contiguous() for i in range(G))

    def three(*ls, residual):
        return tuple(lowrank_dynamic_convolution(*ls[4 * i:4 * i + 4], residual=residual) for i in range(G))

    ds3 = DeviceStep(args, wl, sep, dy3, three, dev, world, dp_ctx, flush)
    m3 = ds3.measure(steps, local)
    ds3.release()
    fwd_b, bwd_b = algorithmic_bytes(wl)
    peak = _peaks()[0]
    ms, ms3 = m["total_ms"] / steps, m3["total_ms"] / steps
    out = {
        "value": world * B * T * steps / (m["total_ms"] / 1e3) / 1e6,
        "unit": "Mtokens/s (three convolutions per token)",
        "ms_per_step": ms,
        "steps": steps,
        "scaling": "weak",
        "config": {**wl, "G": G, "layout": "x, y [B, T, 3D] (fused QKV projection output); z [B, T, 3R]",
                   "global_batch": B * world, "parallelism": f"dp{world}"},
        "hbm_roofline_frac_step": G * (fwd_b + bwd_b) / (ms / 1e3) / (peak * 1e9),
        "gpu_launches": m["launches"],
        "separate_calls": {"ms_per_step": ms3, "gpu_launches": m3["launches"],
                           "hbm_roofline_frac_step": G * (fwd_b + bwd_b) / (ms3 / 1e3) / (peak * 1e9)},
        "speedup_vs_separate": ms3 / ms,
        "clocks": m["clocks"],
    }
    del leaves, sep, ds, ds3
    torch.cuda.empty_cache()
    return out


def run_ours(args, wl: dict) -> None:
    import torch
    import torch.distributed as dist

    from dynamic_conv1d_b200 import headwise_dynamic_convolution, lowrank_dynamic_convolution

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)

    B, T, D, W = wl["B"], wl["T"], wl["D"], wl["W"]
    ntok = B * T
    a = make_inputs_np(wl, seed=100 + rank)
    a_sw = make_inputs_np(wl, rows=1, T=1, seed=7)  # shared parameters identical on all ranks
    bf = torch.bfloat16

    def dev_t(arr, grad=False):
        t = torch.from_numpy(arr).to(dev, bf)
        return t.requires_grad_() if grad else t

    x = dev_t(a["x"], True)
    dy = dev_t(a["dy"])
    if wl["kind"] == "lowrank":
        leaves = [x, dev_t(a["z"], True), dev_t(a_sw["U"], True), dev_t(a_sw["static_w"], True)]
        fn = lowrank_dynamic_convolution
    else:
        leaves = [x, dev_t(a["weight"], True), dev_t(a_sw["static_w"], True)]
        fn = headwise_dynamic_convolution

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    dp_ctx = _dp_ctx_factory(world)

    # ---- the headline step: fwd+bwd of the metric's config
    ds = DeviceStep(args, wl, leaves, dy, fn, dev, world, dp_ctx, flush)
    m = ds.measure(args.steps, local)
    total_ms = m["total_ms"]
    value = world * ntok * args.steps / (total_ms / 1e3) / 1e6

    # ---- dominant kernel: the backward C-ABI call, timed alone (CUDA events)
    roof = kernel_roofline(args, wl, leaves, dy, fn, flush, dev, workload=args.workload)
    graph_on = ds.graph is not None
    graph_error = ds.graph_error
    ds.release()

    # ---- e2e through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        e2e = end_to_end(args, wl, a, a_sw, fn, dev, world)
    del leaves, dy, x, a
    torch.cuda.empty_cache()

    # ---- the other BASELINE configs, device-timed the same way (every rank takes part)
    subs = {}
    if not args.no_sub and args.workload == "lowrank" and args.batch is None and args.seq is None:
        for name in ("headwise_hs32", "headwise_hs1"):
            subs[name] = sub_workload(args, name, dict(WORKLOADS[name]), dev, world, local, rank, flush, "weak")
        # B = 64 split over the ranks (strong scaling: the job's work is fixed)
        cfg5 = dict(WORKLOADS["lowrank_dp"])
        cfg5["B"] = max(1, 64 // world)
        subs["lowrank_dp_cfg5"] = sub_workload(args, "lowrank_dp", cfg5, dev, world, local, rank, flush, "strong")
        subs["lowrank_qkv_cfg4"] = qkv_workload(args, dev, world, local, rank, flush)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(wl)

    if world > 1:
        dist.barrier()
    if rank == 0:
        fwd_b, bwd_b = algorithmic_bytes(wl)
        line = {
            "metric": METRIC,
            "value": value,
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded torch.randn / rand, BASELINE shapes and distributions)",
            "config": {
                "workload": args.workload,
                **wl,
                "global_batch": wl["B"] * world,
                "seq_len": T,
                "parallelism": f"dp{world}",
                "l2": "flushed between steps (256 MiB write outside the timed events)",
                "step": "fwd+bwd, CUDA-graph replay" if graph_on else "fwd+bwd, eager",
                "wall_s_timed_region": m["wall"],
                "hbm_roofline_ms_per_step": (fwd_b + bwd_b) / (_peaks()[0] * 1e9) * 1e3,
                "hbm_roofline_frac_step": ((fwd_b + bwd_b) / (total_ms / args.steps / 1e3)) / (_peaks()[0] * 1e9),
            },
            "roofline": roof,
            "clocks": m["clocks"],
            "gpu_launches": m["launches"],
        }
        if not graph_on and not args.no_graph:
            line["config"]["graph_error"] = graph_error
        if e2e is not None:
            line["e2e"] = e2e
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if subs:
            line["workloads"] = subs
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def kernel_roofline(args, wl, leaves, dy, fn, flush, dev, workload=None) -> dict:
    """Average duration of the lowrank/headwise backward C-ABI call (main kernel +
    its fixed-order reduction pass) and of the forward call, each bracketed by CUDA
    events on the launching stream, L2 flushed before every launch."""
    import torch

    from dynamic_conv1d_b200 import _lib

    lib = _lib.load()
    B, T, D, W = wl["B"], wl["T"], wl["D"], wl["W"]
    st = torch.cuda.current_stream(dev)
    stream = ctypes_stream(st)
    x = leaves[0].detach()
    y = torch.empty_like(x)
    dx = torch.empty_like(x)
    if wl["kind"] == "lowrank":
        z, U, sw = (l.detach() for l in leaves[1:])
        R = z.shape[-1]
        Rk = R + 1
        dz = torch.empty_like(z)
        dU = torch.empty_like(U)
        dsw = torch.empty_like(sw)
        acc = torch.empty(Rk, W * D, device=dev, dtype=torch.float32)
        nb = lib.dynconv_lr_bwd_workspace_bytes(B, T, D, R, W, 0, 1)
        ws = torch.empty(max(nb, 1), device=dev, dtype=torch.uint8)
        nbf = lib.dynconv_lr_fwd_workspace_bytes(B, T, D, R, W, 0, 1)
        wsf = torch.empty(max(nbf, 1), device=dev, dtype=torch.uint8)
        P = _lib.ptr

        def fwd():
            return lib.dynconv_lr_fwd(P(x), P(z), P(U), P(sw), P(y), P(wsf), wsf.numel(), B, T, D, R, W, 0, 1, stream)

        def bwd():
            return lib.dynconv_lr_bwd(P(x), P(z), P(U), P(sw), P(dy), P(dx), P(dz), P(dU), P(dsw), P(acc), P(ws),
                                      ws.numel(), B, T, D, R, W, 0, 1, stream)
    else:
        wgt, sw = (l.detach() for l in leaves[1:])
        H = wgt.shape[2]
        dw = torch.empty_like(wgt)
        dsw = torch.empty_like(sw)
        acc = torch.empty(W, D, device=dev, dtype=torch.float32)
        nb = lib.dynconv_hw_bwd_workspace_bytes(B, T, D, H, W, 0, 1)
        ws = torch.empty(max(nb, 1), device=dev, dtype=torch.uint8)
        P = _lib.ptr

        def fwd():
            return lib.dynconv_hw_fwd(P(x), P(wgt), P(sw), P(y), B, T, D, H, W, 0, 1, stream)

        def bwd():
            return lib.dynconv_hw_bwd(P(x), P(wgt), P(sw), P(dy), P(dx), P(dw), P(dsw), P(acc), P(ws), ws.numel(),
                                      B, T, D, H, W, 0, 1, stream)

    def timed(f, n):
        for _ in range(3):
            _lib.check(f())
        evs = []
        for _ in range(n):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            _lib.check(f())
            e1.record(st)
            evs.append((e0, e1))
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in evs) / n

    n = max(10, args.steps)
    t_fwd = timed(fwd, n)
    t_bwd = timed(bwd, n)
    _lib.check_device(x)
    fwd_b, bwd_b = algorithmic_bytes(wl)
    peak, src = _peaks()
    ach = bwd_b / (t_bwd / 1e3) / 1e9
    ach_f = fwd_b / (t_fwd / 1e3) / 1e9
    return {
        "kernel": f"{wl['kind']} backward (dynconv_{'lr' if wl['kind'] == 'lowrank' else 'hw'}_bwd: main kernel + fixed-order reduction)",
        "bound": "hbm",
        "achieved": ach,
        "peak": peak,
        "peak_source": src,
        "unit": "GB/s",
        "frac": ach / peak,
        "traffic": _traffic_from_profiles(workload or args.workload),
        "algorithmic_bytes_per_launch": bwd_b,
        "ms_per_launch": t_bwd,
        "forward": {"achieved": ach_f, "frac": ach_f / peak, "ms_per_launch": t_fwd, "algorithmic_bytes_per_launch": fwd_b},
    }


def ctypes_stream(st):
    import ctypes

    return ctypes.c_void_p(st.cuda_stream)


def end_to_end(args, wl, a, a_sw, fn, dev, world) -> dict:
    """Public API with pinned host buffers: H2D of x, z/weight, dy; fwd+bwd; D2H of
    y and every gradient; all inside the CUDA-event-timed region.

    The step is pipelined over batch rows on three streams -- uploads of row i+1
    and downloads of row i-1 overlap the fwd+bwd of row i (PCIe is full duplex) --
    and the shared gradients (dU, dstatic_w) accumulate over the rows as autograd
    does for any split batch.  With N ranks the accumulated shared gradients are
    summed over the ranks by one all-reduce per step, then copied back."""
    import torch

    bf = torch.bfloat16
    host = {k: torch.from_numpy(v).to(bf).pin_memory() for k, v in a.items() if k in ("x", "dy", "z", "weight")}
    U = torch.from_numpy(a_sw["U"]).to(dev, bf).requires_grad_() if wl["kind"] == "lowrank" else None
    sw = torch.from_numpy(a_sw["static_w"]).to(dev, bf).requires_grad_()
    second = "z" if wl["kind"] == "lowrank" else "weight"
    outs = {
        "y": torch.empty_like(host["x"]).pin_memory(),
        "dx": torch.empty_like(host["x"]).pin_memory(),
        "d2": torch.empty_like(host[second]).pin_memory(),
        "dsw": torch.empty(sw.shape, dtype=bf).pin_memory(),
    }
    if U is not None:
        outs["dU"] = torch.empty(U.shape, dtype=bf).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = sum(t.numel() * t.element_size() for t in outs.values())
    res = bool(wl["residual"])
    comp = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    rows = wl["B"]
    shared = [p for p in (U, sw) if p is not None]

    def step():
        for p in shared:
            p.grad = None
        for r in range(rows):
            sl = slice(r, r + 1)
            with torch.cuda.stream(s_in):
                x = host["x"][sl].to(dev, non_blocking=True)
                s2 = host[second][sl].to(dev, non_blocking=True)
                dy = host["dy"][sl].to(dev, non_blocking=True)
            comp.wait_stream(s_in)
            for t in (x, s2, dy):
                t.record_stream(comp)
            x.requires_grad_()
            s2.requires_grad_()
            args_ = [x, s2, U, sw] if U is not None else [x, s2, sw]
            y = fn(*args_, residual=res)
            y.backward(dy)
            s_out.wait_stream(comp)
            with torch.cuda.stream(s_out):
                for t in (y, x.grad, s2.grad):
                    t.record_stream(s_out)
                outs["y"][sl].copy_(y.detach(), non_blocking=True)
                outs["dx"][sl].copy_(x.grad, non_blocking=True)
                outs["d2"][sl].copy_(s2.grad, non_blocking=True)
        if world > 1:
            # one collective per step: the rank-local sums of the shared gradients
            import torch.distributed as dist

            flat = torch.cat([p.grad.float().flatten() for p in shared])
            dist.all_reduce(flat, op=dist.ReduceOp.SUM)
            off = 0
            for p in shared:
                n = p.grad.numel()
                p.grad.copy_(flat[off:off + n].view_as(p.grad))
                off += n
        s_out.wait_stream(comp)
        with torch.cuda.stream(s_out):
            outs["dsw"].copy_(sw.grad, non_blocking=True)
            if U is not None:
                outs["dU"].copy_(U.grad, non_blocking=True)
        comp.wait_stream(s_out)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    # Three timed batches of n steps, the fastest kept: the PCIe copies share the
    # host with other tenants, and a transient stall should not stand for the
    # path's throughput.  Every batch holds all of its steps' copies.
    n = max(3, min(args.steps, 10))
    ms = float("inf")
    for _ in range(3):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(comp)
        for _ in range(n):
            step()
        e1.record(comp)
        torch.cuda.synchronize()
        ms = min(ms, e0.elapsed_time(e1) / n)
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    ntok = wl["B"] * wl["T"] * world
    # PCIe rate per direction seen by this rank (bytes of the step / step time)
    return {"value": ntok / (ms / 1e3) / 1e6, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": ms, "steps": n, "batches": "best of 3 batches of `steps` steps",
            "h2d_gbs_per_rank": h2d / (ms / 1e3) / 1e9, "d2h_gbs_per_rank": d2h / (ms / 1e3) / 1e9,
            "collectives_per_step": 1 if world > 1 else 0,
            "pipeline": f"{rows} batch rows per step, upload / compute / download streams"}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="lowrank")
    ap.add_argument("--batch", type=int, default=None, help="override the per-GPU batch (small ncu captures)")
    ap.add_argument("--seq", type=int, default=None, help="override T (small ncu captures)")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sub", action="store_true", help="skip the other BASELINE configs' sub-objects")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    wl = dict(WORKLOADS[args.workload])
    if args.batch:
        wl["B"] = args.batch
    if args.seq:
        wl["T"] = args.seq
    if args.impl == "reference":
        run_reference_arm(args, wl)
    else:
        run_ours(args, wl)


if __name__ == "__main__":
    main()
