"""Headwise dynamic short convolution -- drop-in for ``headwise.py`` of
OliverSieberling/dynamic-conv1d, backed by libdynconv (sm_100a CUDA kernels).

Same public function, same ``torch.autograd.Function`` structure, same argument
meaning and the same ``assert`` preconditions as the reference
(``headwise.py:218-337``); the Triton launches are replaced by calls into the
C ABI (``dynconv_hw_fwd`` / ``dynconv_hw_bwd``).
"""
from __future__ import annotations

import torch

from . import _lib
from .parallel import allreduce_shared_grad, current_group


class _HeadwiseDynamicConvolutionFn(torch.autograd.Function):
    """Mirrors ``_HeadwiseDynamicConvolutionFn`` (headwise.py:218-309)."""

    @staticmethod
    @_lib.on_device
    def forward(ctx, x, weight, static_w, residual):
        B, T, D = x.shape
        H = weight.shape[2]
        W = weight.shape[-1]
        assert D % H == 0, f"D={D} must be divisible by H={H}"
        lib = _lib.load()
        code = _lib.dtype_code(x.dtype)
        # The reference reads weight with contiguous [B,T,H,W] strides
        # (headwise.py:60); make that explicit.  It is cast to x.dtype for the
        # kernel; its gradient is cast back to weight.dtype.
        w_k = weight.to(dtype=x.dtype).contiguous()
        y = torch.empty_like(x)
        _lib.check(
            lib.dynconv_hw_fwd(
                _lib.ptr(x), _lib.ptr(w_k), _lib.ptr(static_w), _lib.ptr(y),
                B, T, D, H, W, code, int(bool(residual)), _lib.stream_of(x),
            )
        )
        _lib.after_call(y)
        ctx.save_for_backward(x, w_k, static_w)
        ctx.weight_dtype = weight.dtype
        ctx.residual = bool(residual)
        ctx.group = current_group()
        return y

    @staticmethod
    @_lib.on_device
    def backward(ctx, dy):
        dy = dy.contiguous()
        x, w_k, static_w = ctx.saved_tensors
        B, T, D = x.shape
        H, W = w_k.shape[2], w_k.shape[3]
        lib = _lib.load()
        code = _lib.dtype_code(x.dtype)
        if dy.dtype != x.dtype:
            dy = dy.to(x.dtype)
        dx = torch.empty_like(x)
        dw = torch.empty((B, T, H, W), device=x.device, dtype=x.dtype)
        has_static = static_w is not None
        dsw = dsw_f32 = ws = None
        if has_static:
            dsw_f32 = torch.empty((W, D), device=x.device, dtype=torch.float32)
            if ctx.group is None:
                dsw = torch.empty((W, D), device=x.device, dtype=static_w.dtype)
            nbytes = lib.dynconv_hw_bwd_workspace_bytes(B, T, D, H, W, code, 1)
            ws = torch.empty(max(int(nbytes), 1), device=x.device, dtype=torch.uint8)
        stream = _lib.stream_of(x)
        _lib.check(
            lib.dynconv_hw_bwd(
                _lib.ptr(x), _lib.ptr(w_k), _lib.ptr(static_w), _lib.ptr(dy),
                _lib.ptr(dx), _lib.ptr(dw), _lib.ptr(dsw), _lib.ptr(dsw_f32),
                _lib.ptr(ws), 0 if ws is None else ws.numel(),
                B, T, D, H, W, code, int(ctx.residual), stream,
            )
        )
        if has_static and ctx.group is not None:
            allreduce_shared_grad(dsw_f32, ctx.group)
            dsw = torch.empty((W, D), device=x.device, dtype=static_w.dtype)
            _lib.check(lib.dynconv_cast_f32(_lib.ptr(dsw_f32), _lib.ptr(dsw), W * D,
                                            _lib.dtype_code(static_w.dtype), stream))
        _lib.after_call(dx)
        if ctx.weight_dtype != dw.dtype:
            dw = dw.to(ctx.weight_dtype)
        return dx, dw, dsw, None


def headwise_dynamic_convolution(
    x: torch.Tensor,
    weight: torch.Tensor,
    static_w: torch.Tensor | None = None,
    residual: bool = False,
) -> torch.Tensor:
    """Headwise dynamic causal short convolution, with optional fused static filter.

    Args:
        x:        [B, T, D] input activations (bfloat16 or float32, CUDA, contiguous).
        weight:   [B, T, H, W] per-token (dynamic) weights; each head spans D // H
                  consecutive channels (D // H must be a power of two).
        static_w: [W, D] optional per-channel static filter added to the dynamic
                  weight at every (b, t).
        residual: add x to the output.

    Returns:
        y: [B, T, D] with y[b,t,d] = sum_w (weight[b,t,d//hs,w] + static_w[w,d]) * x[b,t-w,d]
        (+ x[b,t,d] if residual).  Causal: x[b, t-w] is zero for t < w.

    Same preconditions as the reference (headwise.py:332-336).
    """
    assert x.is_cuda and x.is_contiguous()
    if static_w is not None:
        assert static_w.is_cuda and static_w.is_contiguous()
        assert static_w.dtype == x.dtype
        assert static_w.shape == (weight.shape[-1], x.shape[-1])
    return _HeadwiseDynamicConvolutionFn.apply(x, weight, static_w, residual)
