"""Sequence parallelism for the dynamic convolutions: the time axis is split across
ranks, and each rank exchanges a (W-1)-row halo with its neighbours.

Output step t depends on x at steps t-W+1 .. t only (causal, reference.py:5-39),
so a rank that holds steps [t0, t1) of every sequence needs just the W-1 rows of x
before t0, held by the previous rank.  The forward prepends them (zeros on rank 0,
where they are the sequence's own zero padding), runs the op on the extended
slice and drops the W-1 extra outputs.  In the backward, the gradient that falls
on the borrowed rows is sent back to the previous rank and added to the
gradient of its last W-1 rows.  The mixing weights (z, or the headwise weights)
are needed at the local steps only; the borrowed rows get zero weights, and
their outputs are discarded.  The shared parameters' gradients (U, static_w) are
partial sums over the local steps and are all-reduced through
``data_parallel(group)``, as for batch sharding.

Every rank must hold at least W-1 steps.  Ranks are ordered along time by
their rank in ``group``."""
from __future__ import annotations

import torch
import torch.distributed as dist

from .headwise import headwise_dynamic_convolution
from .lowrank import lowrank_dynamic_convolution
from .parallel import data_parallel


def _peer(group, r: int) -> int:
    return dist.get_global_rank(group, r) if group is not None and group is not dist.group.WORLD else r


def _exchange(send: torch.Tensor | None, send_to: int | None, recv_shape, recv_from: int | None, like: torch.Tensor,
              group) -> torch.Tensor:
    """Posts the send and the receive together (no ordering deadlock) and waits for both."""
    recv = torch.zeros(recv_shape, dtype=like.dtype, device=like.device)
    ops = []
    if send_to is not None:
        ops.append(dist.P2POp(dist.isend, send, _peer(group, send_to), group))
    if recv_from is not None:
        ops.append(dist.P2POp(dist.irecv, recv, _peer(group, recv_from), group))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()
    return recv


def _check_lengths(T: int, h: int, device, group) -> None:
    """Every rank must hold at least h = W-1 steps.  The shortest slice is agreed on
    by a MIN all-reduce before any point-to-point exchange, so that all ranks raise
    together instead of some of them waiting on a halo that never comes."""
    t = torch.tensor([T], dtype=torch.int64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MIN, group=group)
    t_min = int(t.item())
    if t_min < h:
        raise ValueError(f"sequence parallel: each rank needs at least W-1={h} steps; "
                         f"the shortest slice holds {t_min} (this rank {T})")


class _HaloPrepend(torch.autograd.Function):
    """[B, T, D] -> [B, h + T, D]: the previous rank's last h rows, then the local rows."""

    @staticmethod
    def forward(ctx, x, h, group):
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        B, T = x.shape[0], x.shape[1]
        _check_lengths(T, h, x.device, group)
        send = x[:, T - h:].contiguous()
        halo = _exchange(send, rank + 1 if rank + 1 < world else None, (B, h) + tuple(x.shape[2:]),
                         rank - 1 if rank > 0 else None, x, group)
        ctx.h, ctx.group, ctx.T = h, group, T
        return torch.cat([halo, x], dim=1)

    @staticmethod
    def backward(ctx, g):
        h, group, T = ctx.h, ctx.group, ctx.T
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        g = g.contiguous()
        g_halo = g[:, :h].contiguous()
        back = _exchange(g_halo, rank - 1 if rank > 0 else None, g_halo.shape, rank + 1 if rank + 1 < world else None,
                         g, group)
        g_local = g[:, h:].clone()
        if rank + 1 < world:
            g_local[:, T - h:] += back
        return g_local, None, None


def _zero_rows_front(t: torch.Tensor, h: int) -> torch.Tensor:
    pad = torch.zeros((t.shape[0], h) + tuple(t.shape[2:]), dtype=t.dtype, device=t.device)
    return torch.cat([pad, t], dim=1)


def sequence_parallel(fn, x, mix, *params, residual: bool = False, W: int, group=None):
    """Runs ``fn(x_ext, mix_ext, *params, residual=...)`` on this rank's time slice.

    ``mix`` is the per-step mixing input (lowrank z [B, T, R], headwise weight
    [B, T, H, W]); ``params`` are the shared parameters.  Returns the local
    output [B, T, D]; gradients flow to x, mix and params, with the shared ones
    all-reduced over ``group``."""
    group = group if group is not None else dist.group.WORLD
    h = W - 1
    if h == 0:
        with data_parallel(group):
            return fn(x, mix, *params, residual=residual)
    x_ext = _HaloPrepend.apply(x, h, group)
    mix_ext = _zero_rows_front(mix, h)
    with data_parallel(group):
        y_ext = fn(x_ext.contiguous(), mix_ext.contiguous(), *params, residual=residual)
    return y_ext[:, h:]


def lowrank_dynamic_convolution_sp(x, z, U, static_w=None, residual: bool = False, group=None):
    """``lowrank_dynamic_convolution`` with the time axis split over ``group``."""
    W = U.shape[-1] // x.shape[-1]
    return sequence_parallel(lowrank_dynamic_convolution, x, z, U, static_w, residual=residual, W=W, group=group)


def headwise_dynamic_convolution_sp(x, weight, static_w=None, residual: bool = False, group=None):
    """``headwise_dynamic_convolution`` with the time axis split over ``group``."""
    W = weight.shape[-1]
    return sequence_parallel(headwise_dynamic_convolution, x, weight, static_w, residual=residual, W=W, group=group)
