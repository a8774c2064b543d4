"""Low-rank dynamic short convolution -- drop-in for ``lowrank.py`` of
OliverSieberling/dynamic-conv1d, backed by libdynconv (sm_100a CUDA kernels).

Same public function, same ``torch.autograd.Function`` structure, same argument
meaning and the same ``assert`` preconditions as the reference
(``lowrank.py:214-338``).  Differences that a caller can observe only as
"more general" or "less memory traffic":

* the static filter is folded in as rank R inside the kernels; ``U`` is never
  concatenated with ``static_w`` (the reference builds ``F.pad(z)`` and
  ``torch.cat([U, static_w])``, lowrank.py:222-226); on the bf16 tensor-core path
  ``z`` plus the static rank is packed once per call into a small workspace in the
  layout the TMA unit places directly into the MMA operand;
* the returned ``dz`` / ``dU`` are dense tensors of the caller's shapes (the
  reference returns slices of padded buffers, lowrank.py:295-299);
* the dU / dstatic_w reduction is deterministic (fixed-order two-pass; the
  reference uses fp32 atomics, lowrank.py:137).
"""
from __future__ import annotations

import torch

from . import _lib
from .parallel import allreduce_shared_grad, comm_for, current_group


def _fused_dp_backward(lib, group, x, z, U, static_w, dy, dx, dz, dU_f32, ws, B, T, D, R, W, G, code, residual,
                       zpack, stream):
    """The backward with the sum over data-parallel ranks done inside the kernel
    (dynconv_lr_bwd_grouped_dp).  Returns (dU [G*R, W*D], dstatic_w [G, W*D] or None),
    bf16, already summed over the ranks; None when the fused path does not apply
    (single rank, not bf16, outside the tensor-core envelope), and the caller
    all-reduces through torch.distributed."""
    has_static = static_w is not None
    Rk = R + (1 if has_static else 0)
    # The choice must be the same on every rank (they all take part in one exchange),
    # so it rests only on what all ranks share: dtype, W, R_kernel, D, G.
    if x.dtype != torch.bfloat16 or not (1 <= W <= 4) or Rk > 32 or D % 8 != 0 or (G > 1 and D % 128 != 0):
        return None
    if (G * D + 127) // 128 > torch.cuda.get_device_properties(x.device).multi_processor_count:
        return None
    comm = comm_for(group, x.device, G * Rk * W * D)
    if comm is None:
        return None
    dU = torch.empty((G * R, W * D), device=x.device, dtype=x.dtype)
    dsw = torch.empty((G, W * D), device=x.device, dtype=x.dtype) if has_static else None
    status = lib.dynconv_lr_bwd_grouped_dp(
        _lib.ptr(x), _lib.ptr(z), _lib.ptr(U), _lib.ptr(static_w), _lib.ptr(dy),
        _lib.ptr(dx), _lib.ptr(dz), _lib.ptr(dU), _lib.ptr(dsw), _lib.ptr(dU_f32),
        _lib.ptr(ws), ws.numel(), B, T, D, R, W, G, code, int(residual), _lib.ptr(zpack), comm.ptr, stream,
    )
    # Every rank is now committed to the in-kernel exchange: a rank-local refusal (an
    # unaligned tensor, an empty shard) is an error, not a silent switch to NCCL that
    # the other ranks would not make.
    _lib.check(status)
    return dU, dsw


class _LowrankDynamicConvolutionFn(torch.autograd.Function):
    """Mirrors ``_LowrankDynamicConvolutionFn`` (lowrank.py:214-299)."""

    @staticmethod
    @_lib.on_device
    def forward(ctx, x, z, U, static_w, residual):
        B, T, D = x.shape
        R = z.shape[-1]
        W = U.shape[-1] // D
        lib = _lib.load()
        code = _lib.dtype_code(x.dtype)
        # The kernels compute in x.dtype; parameters of another dtype are cast
        # for the call and their gradients cast back.
        z_k = z if z.dtype == x.dtype else z.to(x.dtype)
        U_k = U if U.dtype == x.dtype else U.to(x.dtype)
        sw_k = static_w if (static_w is None or static_w.dtype == x.dtype) else static_w.to(x.dtype)
        y = torch.empty_like(x)
        nbytes = lib.dynconv_lr_fwd_workspace_bytes(B, T, D, R, W, code, int(static_w is not None))
        ws = torch.empty(max(int(nbytes), 1), device=x.device, dtype=torch.uint8)
        _lib.check(
            lib.dynconv_lr_fwd(
                _lib.ptr(x), _lib.ptr(z_k), _lib.ptr(U_k), _lib.ptr(sw_k), _lib.ptr(y),
                _lib.ptr(ws), ws.numel(),
                B, T, D, R, W, code, int(bool(residual)), _lib.stream_of(x),
            )
        )
        _lib.after_call(y)
        ctx.save_for_backward(x, z_k, U_k, sw_k)
        ctx.zpack = ws if nbytes > 0 else None  # z packed for the tensor cores, reused by the backward
        ctx.dtypes = (z.dtype, U.dtype, None if static_w is None else static_w.dtype)
        ctx.residual = bool(residual)
        ctx.group = current_group()
        return y

    @staticmethod
    @_lib.on_device
    def backward(ctx, dy):
        dy = dy.contiguous()
        x, z, U, static_w = ctx.saved_tensors
        B, T, D = x.shape
        R = z.shape[-1]
        W = U.shape[-1] // D
        has_static = static_w is not None
        Rk = R + (1 if has_static else 0)
        lib = _lib.load()
        code = _lib.dtype_code(x.dtype)
        if dy.dtype != x.dtype:
            dy = dy.to(x.dtype)
        dx = torch.empty_like(x)
        dz = torch.empty_like(z)
        dU_f32 = torch.empty((Rk, W * D), device=x.device, dtype=torch.float32)
        nbytes = lib.dynconv_lr_bwd_workspace_bytes(B, T, D, R, W, code, int(has_static))
        ws = torch.empty(max(int(nbytes), 1), device=x.device, dtype=torch.uint8)
        stream = _lib.stream_of(x)
        reduce_first = ctx.group is not None
        fused = None
        if reduce_first:
            fused = _fused_dp_backward(lib, ctx.group, x, z, U, static_w, dy, dx, dz, dU_f32, ws,
                                       B, T, D, R, W, 1, code, ctx.residual, ctx.zpack, stream)
        if fused is not None:
            reduce_first = False  # summed over the ranks and cast inside the kernel
            dU = fused[0]
            dsw = fused[1].view(W, D) if has_static else None
        else:
            dU = None if reduce_first else torch.empty_like(U)
            dsw = None if (reduce_first or not has_static) else torch.empty((W, D), device=x.device, dtype=x.dtype)
            _lib.check(
                lib.dynconv_lr_bwd_grouped(
                    _lib.ptr(x), _lib.ptr(z), _lib.ptr(U), _lib.ptr(static_w), _lib.ptr(dy),
                    _lib.ptr(dx), _lib.ptr(dz), _lib.ptr(dU), _lib.ptr(dsw), _lib.ptr(dU_f32),
                    _lib.ptr(ws), ws.numel(),
                    B, T, D, R, W, 1, code, int(ctx.residual), _lib.ptr(ctx.zpack), stream,
                )
            )
        if reduce_first:
            allreduce_shared_grad(dU_f32, ctx.group)
            # one cast of the reduced accumulator; dU and dstatic_w are row views of it
            # (the reference also returns slices of one buffer, lowrank.py:295-299)
            g = torch.empty((Rk, W * D), device=x.device, dtype=x.dtype)
            _lib.check(lib.dynconv_cast_f32(_lib.ptr(dU_f32), _lib.ptr(g), Rk * W * D, code, stream))
            dU = g[:R]
            if has_static:
                dsw = g[R].view(W, D)
        _lib.after_call(dx)
        z_dt, U_dt, sw_dt = ctx.dtypes
        if dz.dtype != z_dt:
            dz = dz.to(z_dt)
        if dU.dtype != U_dt:
            dU = dU.to(U_dt)
        if dsw is not None and dsw.dtype != sw_dt:
            dsw = dsw.to(sw_dt)
        return dx, dz, dU, dsw, None


def lowrank_dynamic_convolution(
    x: torch.Tensor,
    z: torch.Tensor,
    U: torch.Tensor,
    static_w: torch.Tensor | None = None,
    residual: bool = False,
) -> torch.Tensor:
    """Low-rank dynamic short convolution, with optional fused static filter.

    The dynamic weights ``z @ U`` are generated on chip (tensor cores for bf16)
    and never written to HBM.

    Args:
        x:        [B, T, D] input activations (bfloat16 or float32, CUDA, contiguous).
        z:        [B, T, R] hidden states after the first projection.
        U:        [R, W*D] second projection, viewed as (R, W, D).
        static_w: [W, D] optional static filter, fused as one extra rank, so
                  R+1 must be a power of two when it is given (R otherwise).
        residual: add x to the output.

    Returns:
        y: [B, T, D] with y[b,t,d] = sum_w (sum_r z[b,t,r] U[r,w*D+d] + static_w[w,d]) * x[b,t-w,d]
        (+ x[b,t,d] if residual).

    Same preconditions as the reference (lowrank.py:328-337).
    """
    assert x.is_cuda and x.is_contiguous()
    assert z.is_cuda and z.is_contiguous()
    assert U.is_cuda and U.is_contiguous()
    R = z.shape[-1]
    R_kernel = R + 1 if static_w is not None else R
    assert R_kernel & (R_kernel - 1) == 0, "rank R must be a power of 2. If static_w is set R+1 must be a power of 2."
    if static_w is not None:
        assert static_w.is_cuda and static_w.is_contiguous()
        assert static_w.dtype == z.dtype == U.dtype
        assert static_w.shape == (U.shape[-1] // x.shape[-1], x.shape[-1])
    return _LowrankDynamicConvolutionFn.apply(x, z, U, static_w, residual)


class _LowrankGroupedFn(torch.autograd.Function):
    """G lowrank convolutions in one launch per direction (``dynconv_lr_fwd_grouped``
    / ``dynconv_lr_bwd_grouped``): x [B,T,G*D], z [B,T,G*R], U [G,R,W*D],
    static_w [G,W,D].  bf16 tensor-core path only; ``lowrank_dynamic_convolution_grouped``
    checks the envelope and otherwise runs the groups one by one."""

    @staticmethod
    @_lib.on_device
    def forward(ctx, x, z, U, static_w, residual):
        B, T, Dt = x.shape
        G, R = U.shape[0], U.shape[1]
        D = Dt // G
        W = U.shape[-1] // D
        lib = _lib.load()
        code = _lib.dtype_code(x.dtype)
        y = torch.empty_like(x)
        has_static = static_w is not None
        nbytes = lib.dynconv_lr_fwd_grouped_workspace_bytes(B, T, D, R, W, G, code, int(has_static))
        ws = torch.empty(max(int(nbytes), 1), device=x.device, dtype=torch.uint8)
        _lib.check(
            lib.dynconv_lr_fwd_grouped(
                _lib.ptr(x), _lib.ptr(z), _lib.ptr(U), _lib.ptr(static_w), _lib.ptr(y),
                _lib.ptr(ws), ws.numel(),
                B, T, D, R, W, G, code, int(bool(residual)), _lib.stream_of(x),
            )
        )
        _lib.after_call(y)
        ctx.save_for_backward(x, z, U, static_w)
        ctx.zpack = ws if nbytes > 0 else None  # z packed for the tensor cores, reused by the backward
        ctx.residual = bool(residual)
        ctx.group = current_group()
        return y

    @staticmethod
    @_lib.on_device
    def backward(ctx, dy):
        dy = dy.contiguous()
        x, z, U, static_w = ctx.saved_tensors
        B, T, Dt = x.shape
        G, R = U.shape[0], U.shape[1]
        D = Dt // G
        W = U.shape[-1] // D
        has_static = static_w is not None
        Rk = R + (1 if has_static else 0)
        lib = _lib.load()
        code = _lib.dtype_code(x.dtype)
        if dy.dtype != x.dtype:
            dy = dy.to(x.dtype)
        dx = torch.empty_like(x)
        dz = torch.empty_like(z)
        dU_f32 = torch.empty((G, Rk, W * D), device=x.device, dtype=torch.float32)
        nbytes = lib.dynconv_lr_bwd_grouped_workspace_bytes(B, T, D, R, W, G, code, int(has_static))
        ws = torch.empty(max(int(nbytes), 1), device=x.device, dtype=torch.uint8)
        stream = _lib.stream_of(x)
        reduce_first = ctx.group is not None
        if reduce_first:
            fused = _fused_dp_backward(lib, ctx.group, x, z, U, static_w, dy, dx, dz, dU_f32, ws,
                                       B, T, D, R, W, G, code, ctx.residual, ctx.zpack, stream)
            if fused is not None:
                _lib.after_call(dx)
                dsw = fused[1].view(G, W, D) if has_static else None
                return dx, dz, fused[0].view(G, R, W * D), dsw, None
        dU = None if reduce_first else torch.empty_like(U)
        dsw = None if (reduce_first or not has_static) else torch.empty_like(static_w)
        _lib.check(
            lib.dynconv_lr_bwd_grouped(
                _lib.ptr(x), _lib.ptr(z), _lib.ptr(U), _lib.ptr(static_w), _lib.ptr(dy),
                _lib.ptr(dx), _lib.ptr(dz), _lib.ptr(dU), _lib.ptr(dsw), _lib.ptr(dU_f32),
                _lib.ptr(ws), ws.numel(),
                B, T, D, R, W, G, code, int(ctx.residual), _lib.ptr(ctx.zpack), stream,
            )
        )
        if reduce_first:
            # one all-reduce for all G groups' dU and dstatic_w rows
            allreduce_shared_grad(dU_f32, ctx.group)
            g = torch.empty((G, Rk, W * D), device=x.device, dtype=x.dtype)
            _lib.check(lib.dynconv_cast_f32(_lib.ptr(dU_f32), _lib.ptr(g), G * Rk * W * D, code, stream))
            dU = g[:, :R]
            if has_static:
                dsw = g[:, R].view(G, W, D)
        _lib.after_call(dx)
        return dx, dz, dU, dsw, None


def grouped_supported(x: torch.Tensor, D: int, R: int, W: int, G: int, has_static: bool) -> bool:
    """Whether the one-launch grouped kernels take this call (bf16, W <= 4,
    R_kernel <= 32, D % 128 == 0, G*D/128 CTAs co-resident, 16-byte aligned)."""
    Rk = R + (1 if has_static else 0)
    if x.dtype != torch.bfloat16 or not (1 <= W <= 4) or Rk > 32 or D % 128 != 0:
        return False
    props = torch.cuda.get_device_properties(x.device)
    return G * D // 128 <= props.multi_processor_count


def lowrank_dynamic_convolution_grouped(
    x: torch.Tensor,
    z: torch.Tensor,
    U: torch.Tensor,
    static_w: torch.Tensor | None = None,
    residual: bool = False,
) -> torch.Tensor:
    """G low-rank dynamic convolutions side by side -- e.g. the query, key and value
    convolutions of one attention layer (reference README.md:86-105) -- computed
    by one forward and one backward kernel launch.

    Args:
        x:        [B, T, G*D]; group g's input is x[..., g*D:(g+1)*D] (the layout of a
                  fused QKV projection's output, read in place).
        z:        [B, T, G*R]; group g's mixing coefficients are z[..., g*R:(g+1)*R].
        U:        [G, R, W*D], one second projection per group.
        static_w: [G, W, D] optional static filters (one extra rank per group).
        residual: add x to the output.

    Returns:
        y [B, T, G*D] with y[..., g*D:(g+1)*D] =
        lowrank_dynamic_convolution(x_g, z_g, U[g], static_w[g], residual).

    Under ``data_parallel()`` the backward all-reduces one [G, R_kernel, W*D]
    buffer.  Outside the grouped kernels' envelope (see ``grouped_supported``) the
    groups run one by one through ``lowrank_dynamic_convolution``.
    """
    assert x.is_cuda and x.is_contiguous() and z.is_contiguous() and U.is_contiguous()
    G, R = U.shape[0], U.shape[1]
    B, T, Dt = x.shape
    assert Dt % G == 0 and z.shape == (B, T, G * R), "x must be [B,T,G*D] and z [B,T,G*R]"
    D = Dt // G
    W = U.shape[-1] // D
    R_kernel = R + 1 if static_w is not None else R
    assert R_kernel & (R_kernel - 1) == 0, "rank R must be a power of 2. If static_w is set R+1 must be a power of 2."
    if static_w is not None:
        assert static_w.is_contiguous() and static_w.shape == (G, W, D)
        assert static_w.dtype == z.dtype == U.dtype
    if G > 1 and z.dtype == U.dtype == x.dtype and grouped_supported(x, D, R, W, G, static_w is not None):
        return _LowrankGroupedFn.apply(x, z, U, static_w, residual)
    outs = [
        lowrank_dynamic_convolution(
            x[..., g * D:(g + 1) * D].contiguous(), z[..., g * R:(g + 1) * R].contiguous(), U[g],
            None if static_w is None else static_w[g], residual)
        for g in range(G)
    ]
    return torch.cat(outs, dim=-1)
