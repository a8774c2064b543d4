"""Sequence parallelism for the dynamic convolutions: the time axis is split across
ranks, and each rank exchanges a (W-1)-row halo with its neighbours.

Output step t depends on x at steps t-W+1 .. t only (causal, reference.py:5-39),
so a rank that holds steps [t0, t1) of every sequence needs just the W-1 rows of x
before t0, held by the previous rank (on rank 0 they are the sequence's own zero
padding).  The op runs on the local slice unchanged, and a second call on a
2(W-1)-row window supplies the terms of the borrowed rows (``sequence_parallel``
below), so nothing of the size of the slice is copied.  In the backward, the
gradient that falls on the borrowed rows is sent back to the previous rank and
added to the gradient of its last W-1 rows.  The shared parameters' gradients
(U, static_w) are partial sums over the local steps; they are summed over the
ranks by one all-reduce, as for batch sharding.

Every rank must hold at least W-1 steps.  Ranks are ordered along time by
their rank in ``group``."""
from __future__ import annotations

import torch
import torch.distributed as dist

from .headwise import headwise_dynamic_convolution
from .lowrank import lowrank_dynamic_convolution
from .parallel import local_gradients


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


class _SPEnter(torch.autograd.Function):
    """Splits the inputs of one sequence-parallel call into the main call's inputs
    (views of the local tensors) and the halo correction's inputs, and does in its
    backward every exchange the call needs, in one fixed order on every rank: the
    halo gradient back to the previous rank, then one all-reduce of the shared
    gradients.

    Correction inputs, each 2h rows long: x_s = [the previous rank's last h rows of x,
    h zero rows], mix_s = [h zero rows, the first h local rows of mix]."""

    @staticmethod
    def forward(ctx, h, group, x, mix, *params):
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        B, T = x.shape[0], x.shape[1]
        _check_lengths(T, h, x.device, group)
        has_prev, has_next = rank > 0, rank + 1 < world
        send = x[:, T - h:].contiguous() if has_next else None
        halo = _exchange(send, rank + 1 if has_next else None, (B, h) + tuple(x.shape[2:]),
                         rank - 1 if has_prev else None, x, group)
        ctx.h, ctx.group, ctx.T = h, group, T
        ctx.has_prev, ctx.has_next = has_prev, has_next
        ctx.x_meta = (x.shape, x.dtype, x.device)
        x_s = torch.zeros((B, 2 * h) + tuple(x.shape[2:]), dtype=x.dtype, device=x.device)
        x_s[:, :h] = halo
        mix_s = torch.zeros((B, 2 * h) + tuple(mix.shape[2:]), dtype=mix.dtype, device=mix.device)
        mix_s[:, h:] = mix[:, :h]
        return (x.view_as(x), mix.view_as(mix), x_s, mix_s) + tuple(p.view_as(p) for p in params)

    @staticmethod
    def backward(ctx, g_x, g_mix, g_xs, g_mixs, *g_params):
        h, group, T = ctx.h, ctx.group, ctx.T
        rank = dist.get_rank(group)
        shape, dtype, device = ctx.x_meta
        halo_shape = (shape[0], h) + tuple(shape[2:])
        # the gradient of the borrowed rows goes back to their owner, the previous rank
        # (sent even when it is zero: the owner posts the matching receive)
        send = None
        if ctx.has_prev:
            send = (g_xs[:, :h].contiguous() if g_xs is not None
                    else torch.zeros(halo_shape, dtype=dtype, device=device))
        back = _exchange(send, rank - 1 if ctx.has_prev else None, halo_shape,
                         rank + 1 if ctx.has_next else None, torch.empty(0, dtype=dtype, device=device), group)
        # g_x / g_mix are the main call's fresh gradient buffers (one consumer each):
        # the h-row fix-ups are added in place
        if ctx.has_next and g_x is not None:
            g_x[:, T - h:] += back
        if g_mixs is not None and g_mix is not None:
            g_mix[:, :h] += g_mixs[:, h:]
        return (None, None, g_x, g_mix) + _sum_shared(list(g_params), group)


def _sum_shared(grads, group) -> tuple:
    """One SUM all-reduce of the shared parameters' gradients over the ranks (float32,
    packed into one buffer), cast back to each parameter's dtype."""
    live = [g for g in grads if g is not None]
    if not live or dist.get_world_size(group) == 1:
        return tuple(grads)
    flat = torch.cat([g.reshape(-1).float() for g in live])
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    out, i = [], 0
    for g in grads:
        if g is None:
            out.append(None)
            continue
        out.append(flat[i:i + g.numel()].view(g.shape).to(g.dtype))
        i += g.numel()
    return tuple(out)


class _SharedSum(torch.autograd.Function):
    """Identity on the shared parameters; their gradients are summed over the ranks
    (W = 1: no halo, nothing else to exchange)."""

    @staticmethod
    def forward(ctx, group, *params):
        ctx.group = group
        return tuple(p.view_as(p) for p in params)

    @staticmethod
    def backward(ctx, *grads):
        return (None,) + _sum_shared(list(grads), ctx.group)


class _SPExit(torch.autograd.Function):
    """y[:, :h] += the halo correction's last h output rows (in place on the main
    call's output)."""

    @staticmethod
    def forward(ctx, y, y_s, h):
        y[:, :h] += y_s[:, h:]
        ctx.mark_dirty(y)
        ctx.h = h
        return y

    @staticmethod
    def backward(ctx, g):
        h = ctx.h
        g_s = torch.zeros((g.shape[0], 2 * h) + tuple(g.shape[2:]), dtype=g.dtype, device=g.device)
        g_s[:, h:] = g[:, :h]
        return g, g_s, None


def sequence_parallel(fn, x, mix, *params, residual: bool = False, W: int, group=None):
    """Runs ``fn(x, mix, *params, residual=...)`` on this rank's time slice.

    ``mix`` is the per-step mixing input (lowrank z [B, T, R], headwise weight
    [B, T, H, W]); ``params`` are the shared parameters.  Returns the local
    output [B, T, D]; gradients flow to x, mix and params, with the shared ones
    summed over ``group``.

    ``fn`` runs on the local slice as it is -- its first W-1 outputs then miss the
    terms of the previous rank's rows, which the causal window reads as zero padding --
    and once more on a 2(W-1)-row window (the borrowed rows, then zeros as x; zeros,
    then the first W-1 local rows as mix, without the residual).  The op is linear in
    x for fixed mixing weights, so that window's last W-1 outputs are exactly the
    missing terms, and they are added to the first W-1 outputs.  No copy of the
    local slice is made; the extra traffic is O(W) rows per sequence.  Rank 0 has
    no previous rank and skips the window."""
    group = group if group is not None else dist.group.WORLD
    h = W - 1
    live = [p for p in params if p is not None]
    if h == 0:
        live_v = list(_SharedSum.apply(group, *live)) if live else []
    else:
        x, mix, x_s, mix_s, *live_v = _SPEnter.apply(h, group, x, mix, *live)
    it = iter(live_v)
    params_v = [None if p is None else next(it) for p in params]
    # the shared gradients are summed once, by _SPEnter's (or _SharedSum's) backward, not by fn
    with local_gradients():
        y = fn(x, mix, *params_v, residual=residual)
        if h == 0:
            return y
        if dist.get_rank(group) > 0:
            y_s = fn(x_s, mix_s, *params_v, residual=False)
            y = _SPExit.apply(y, y_s, h)
    return y


def lowrank_dynamic_convolution_sp(x, z, U, static_w=None, residual: bool = False, group=None):
    """``lowrank_dynamic_convolution`` with the time axis split over ``group``."""
    W = U.shape[-1] // x.shape[-1]
    return sequence_parallel(lowrank_dynamic_convolution, x, z, U, static_w, residual=residual, W=W, group=group)


def headwise_dynamic_convolution_sp(x, weight, static_w=None, residual: bool = False, group=None):
    """``headwise_dynamic_convolution`` with the time axis split over ``group``."""
    W = weight.shape[-1]
    return sequence_parallel(headwise_dynamic_convolution, x, weight, static_w, residual=residual, W=W, group=group)
