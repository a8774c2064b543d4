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

For the lowrank op on the bf16 tensor-core path the sum over ranks is done
inside the backward kernel itself (``comm_for`` / ``dynconv_lr_bwd_grouped_dp``:
every rank stores its sum into every peer's landing buffer over NVLink and adds
the world's contributions in rank order); everything else all-reduces through
``torch.distributed`` (NCCL) on the current stream.  Outside the context nothing
is reduced, exactly like the single-GPU reference.
"""
from __future__ import annotations

import contextlib
import ctypes
import os
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


@contextlib.contextmanager
def local_gradients():
    """Within this context the ops reduce nothing, even inside ``data_parallel``: the
    caller sums the shared gradients itself (``sequence_parallel`` does, once for its
    two calls)."""
    prev = getattr(_state, "group", None)
    _state.group = None
    try:
        yield
    finally:
        _state.group = prev


class _Comm:
    """The library's data-parallel communicator for one (process group, device): peer
    landing buffers mapped over CUDA IPC, used by the fused lowrank backward
    (``dynconv_lr_bwd_grouped_dp``) instead of an NCCL all-reduce."""

    def __init__(self, group, device: torch.device, cap: int):
        from . import _lib

        lib = _lib.load()
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.cap = cap
        blob = ctypes.create_string_buffer(int(lib.dynconv_comm_blob_bytes()))
        ptr = ctypes.c_void_p()
        with torch.cuda.device(device):
            _lib.check(lib.dynconv_comm_create(self.world, self.rank, cap, ctypes.byref(ptr), blob))
            blobs = [None] * self.world
            dist.all_gather_object(blobs, blob.raw, group=group)
            status = lib.dynconv_comm_connect(ptr, b"".join(blobs))
            # every rank must have mapped its peers before any of them uses the buffers
            flag = torch.tensor([0 if status == 0 else 1], device=device, dtype=torch.int32)
            dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=group)
        if status != 0 or int(flag.item()) != 0:
            lib.dynconv_comm_destroy(ptr)
            _lib.check(status)
            raise RuntimeError("libdynconv: a peer rank could not connect its communicator")
        self.ptr = ptr


_comms: dict = {}


def fused_dp_enabled() -> bool:
    """The fused all-reduce inside the lowrank backward (DYNCONV_DP_FUSED=0 turns it off)."""
    return os.environ.get("DYNCONV_DP_FUSED", "1") not in ("", "0")


def comm_for(group, device: torch.device, nfloats: int) -> "_Comm | None":
    """The communicator of ``group`` on ``device`` holding at least ``nfloats`` floats per
    slot, created collectively on first use (every rank reaches this call with the same
    size, as every rank runs the same backward).  None for a single rank, when the
    fused path is off, or while a CUDA graph is being captured without one."""
    if group is None or not fused_dp_enabled():
        return None
    world = dist.get_world_size(group)
    if world < 2 or world > 8:
        return None
    key = (id(group), device.index)
    c = _comms.get(key)
    if c is not None and c.cap >= nfloats:
        return c
    if torch.cuda.is_current_stream_capturing():
        return None  # no allocation inside a capture; the NCCL path runs instead
    cap = max(1 << 18, (nfloats + 3) // 4 * 4)
    c = _Comm(group, device, cap)
    _comms[key] = c  # an older, smaller communicator stays mapped (peers may still hold it)
    return c


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
