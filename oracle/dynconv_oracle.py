"""CPU oracle for the dynamic short convolution ops (numpy, float32).

TEST INFRASTRUCTURE ONLY. Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
module, and only as the checker or as the timed CPU baseline.  The product path
(``dynamic_conv1d_b200``) never calls it: that path runs the CUDA library or
raises.

What it restates (reference project OliverSieberling/dynamic-conv1d):

* ``headwise_fwd``  follows ``reference.py:5-20``  (headwise_dynamic_convolution_ref)
* ``lowrank_fwd``   follows ``reference.py:23-39`` (lowrank_dynamic_convolution_ref)
* ``headwise_bwd`` / ``lowrank_bwd`` are the gradients that torch autograd takes
  through those two functions (the reference has no hand-written CPU backward; its
  ``test.py:20-30`` obtains them with ``.backward(dy)``).  They are written out
  here analytically.

Math (``README.md:12-17``), lag index ``w``, causal zero padding inside a batch row::

    headwise: y[b,t,d] = sum_w (weight[b,t,d//hs,w] + static_w[w,d]) * x[b,t-w,d]  (+ x[b,t,d])
    lowrank : y[b,t,d] = sum_w ((z@U).view(B,T,W,D)[b,t,w,d] + static_w[w,d]) * x[b,t-w,d]  (+ x)

Pinning: ``tests/golden/*.npz`` hold outputs of the reference's own ``reference.py``
(forward + torch autograd backward), produced by ``tests/golden/make_golden.py``;
``tests/test_oracle.py`` checks this module against every fixture.

All arrays are float32 numpy arrays; results are float32 (the reference computes
in float32 and casts to ``x.dtype`` at the end, ``reference.py:20,39``).  The
parity tests compare the CUDA results against these float32 values.
"""
from __future__ import annotations

import numpy as np

__all__ = [
    "headwise_fwd",
    "headwise_bwd",
    "lowrank_fwd",
    "lowrank_bwd",
    "shift_past",
    "shift_future",
]


def shift_past(a: np.ndarray, k: int) -> np.ndarray:
    """out[:, t] = a[:, t-k] with zeros for t < k (per batch row).

    Restates ``F.pad(x, (0, 0, k, 0))[:, :T, :]`` of ``reference.py:13,35``.
    """
    if k == 0:
        return a
    out = np.zeros_like(a)
    T = a.shape[1]
    if k < T:
        out[:, k:] = a[:, : T - k]
    return out


def shift_future(a: np.ndarray, k: int) -> np.ndarray:
    """out[:, t] = a[:, t+k] with zeros for t+k >= T: the adjoint of ``shift_past``."""
    if k == 0:
        return a
    out = np.zeros_like(a)
    T = a.shape[1]
    if k < T:
        out[:, : T - k] = a[:, k:]
    return out


def _f32(a):
    return None if a is None else np.asarray(a, dtype=np.float32)


def headwise_fwd(x, weight, static_w=None, residual=False):
    """Forward of ``reference.py:5-20``.

    x [B,T,D], weight [B,T,H,W], static_w [W,D] or None -> y [B,T,D] (float32).
    """
    x, weight, static_w = _f32(x), _f32(weight), _f32(static_w)
    B, T, D = x.shape
    H, W = weight.shape[2], weight.shape[3]
    assert D % H == 0, f"D={D} must be divisible by H={H}"
    hs = D // H
    y = np.zeros_like(x)
    for k in range(W):
        x_shift = shift_past(x, k)
        w_tap = np.repeat(weight[:, :, :, k], hs, axis=2)
        if static_w is not None:
            w_tap = w_tap + static_w[k]
        y += w_tap * x_shift
    if residual:
        y += x
    return y


def headwise_bwd(x, weight, static_w, dy, residual=False):
    """Gradients of ``reference.py:5-20`` for upstream gradient ``dy``.

    Returns (dx [B,T,D], dweight [B,T,H,W], dstatic_w [W,D] or None).
    """
    x, weight, static_w, dy = _f32(x), _f32(weight), _f32(static_w), _f32(dy)
    B, T, D = x.shape
    H, W = weight.shape[2], weight.shape[3]
    hs = D // H
    dx = np.zeros_like(x)
    dw = np.zeros((B, T, H, W), dtype=np.float32)
    dsw = np.zeros((W, D), dtype=np.float32) if static_w is not None else None
    for k in range(W):
        w_tap = np.repeat(weight[:, :, :, k], hs, axis=2)
        if static_w is not None:
            w_tap = w_tap + static_w[k]
        # y[t] += w_tap[t] * x[t-k]  =>  dx[t-k] += dy[t] * w_tap[t]
        dx += shift_future(dy * w_tap, k)
        prod = dy * shift_past(x, k)
        dw[:, :, :, k] = prod.reshape(B, T, H, hs).sum(axis=-1)
        if dsw is not None:
            dsw[k] = prod.sum(axis=(0, 1))
    if residual:
        dx += dy
    return dx, dw, dsw


def lowrank_fwd(x, z, U, static_w=None, residual=False):
    """Forward of ``reference.py:23-39``.

    x [B,T,D], z [B,T,R], U [R, W*D], static_w [W,D] or None -> y [B,T,D] (float32).
    """
    x, z, U, static_w = _f32(x), _f32(z), _f32(U), _f32(static_w)
    B, T, D = x.shape
    R, WD = U.shape
    assert WD % D == 0, f"Last dim. of U ({WD}) must be divisible by D={D}"
    W = WD // D
    K = (z.reshape(B * T, R) @ U).reshape(B, T, W, D)
    if static_w is not None:
        K = K + static_w
    y = np.zeros_like(x)
    for k in range(W):
        y += K[:, :, k, :] * shift_past(x, k)
    if residual:
        y += x
    return y


def lowrank_bwd(x, z, U, static_w, dy, residual=False):
    """Gradients of ``reference.py:23-39`` for upstream gradient ``dy``.

    Returns (dx [B,T,D], dz [B,T,R], dU [R,W*D], dstatic_w [W,D] or None).
    """
    x, z, U, static_w, dy = _f32(x), _f32(z), _f32(U), _f32(static_w), _f32(dy)
    B, T, D = x.shape
    R, WD = U.shape
    W = WD // D
    K = (z.reshape(B * T, R) @ U).reshape(B, T, W, D)
    if static_w is not None:
        K = K + static_w
    dx = np.zeros_like(x)
    dK = np.zeros((B, T, W, D), dtype=np.float32)
    for k in range(W):
        dx += shift_future(dy * K[:, :, k, :], k)
        dK[:, :, k, :] = dy * shift_past(x, k)
    if residual:
        dx += dy
    dK2 = dK.reshape(B * T, WD)
    dz = (dK2 @ U.T).reshape(B, T, R)
    dU = z.reshape(B * T, R).T @ dK2
    dsw = dK.sum(axis=(0, 1)) if static_w is not None else None
    return dx, dz, dU, dsw
