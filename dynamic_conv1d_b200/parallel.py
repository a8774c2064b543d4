"""Data parallelism for the dynamic convolution ops: batch sharding plus one
all-reduce of the float32 shared-gradient buffer.

Every output row (b, t) depends only on batch row b, so the batch is split
across ranks and x, z/weight, y and their gradients never cross a GPU boundary.
Only the parameters shared by all rows -- ``U`` and ``static_w`` -- get a
gradient that must be summed over ranks.  Inside ``data_parallel(group)``, the
backward of both ops all-reduces (SUM) their float32 accumulator before the
cast to the parameter dtype:

* lowrank: the packed ``[R_kernel, W*D]`` buffer (dU rows + the folded
  static_w row), one collective per call;
* headwise: the ``[W, D]`` dstatic_w buffer (dweight is per row, no exchange).

The collective runs on the current stream through ``torch.distributed``
(NCCL over NVLink on one B200 node).  Outside the context nothing is reduced,
exactly like the single-GPU reference.
"""
from __future__ import annotations

import contextlib
import threading

import torch
import torch.distributed as dist

_state = threading.local()


def current_group():
    """The process group gradients are reduced over, or None (single process)."""
    return getattr(_state, "group", None)


@contextlib.contextmanager
def data_parallel(group=None):
    """Within this context the backward all-reduces the shared float32 gradient.

    ``group`` defaults to the default process group (``dist.group.WORLD``).
    """
    if not dist.is_available() or not dist.is_initialized():
        raise RuntimeError("data_parallel() needs an initialised torch.distributed process group")
    prev = getattr(_state, "group", None)
    _state.group = group if group is not None else dist.group.WORLD
    try:
        yield _state.group
    finally:
        _state.group = prev


def allreduce_shared_grad(buf: torch.Tensor, group) -> None:
    """SUM-all-reduce a float32 shared-gradient accumulator in place."""
    if group is None:
        return
    if dist.get_world_size(group) > 1:
        dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=group)


def shard_rows(t: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """The contiguous batch shard of ``t`` (dim 0) owned by ``rank``.

    Batch rows are assigned in contiguous blocks; when ``world`` does not divide
    the batch, the first ``B % world`` ranks take one extra row.
    """
    B = t.shape[0]
    base, extra = divmod(B, world)
    start = rank * base + min(rank, extra)
    stop = start + base + (1 if rank < extra else 0)
    return t[start:stop]
