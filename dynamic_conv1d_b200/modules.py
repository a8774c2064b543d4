"""nn.Module wrappers of the low-rank dynamic convolution, as in the reference's
README (README.md:57-84: ``LowRankDynamicShortConvolution``; README.md:86-105:
one module each for the queries, keys and values of an attention layer).

``LowRankDynamicShortConvolution`` has the reference module's parameters, their
initialisation and its error: ``proj_in`` (d_model -> R, no bias) produces z from
the pre-norm input, ``proj_out`` is U (zeros, [R, W*d_model]), and
``proj_out_bias`` is static_w ([W, d_model], uniform in +-1/sqrt(W)), folded into
the kernels as rank R -- so R+1 must be a power of two.

``QKVLowRankDynamicShortConvolution`` holds the three modules' parameters,
computes the three z projections as one GEMM (the three proj_in weights stacked,
one read of the pre-norm activations instead of three) and the three
convolutions as one grouped kernel launch per direction.

proj_in is an ordinary GEMM (cuBLAS through ``torch.nn.functional.linear``): z
needs a dot product over all d_model channels for each token, while a
convolution tile sees 128 of them, so it is not fused into the convolution
kernels."""
from __future__ import annotations

import math

import torch
from torch import nn

from .lowrank import lowrank_dynamic_convolution, lowrank_dynamic_convolution_grouped


def _check_rank(R: int) -> None:
    if ((R + 1) & R) != 0:
        raise ValueError("R+1 must be a power of two")


class LowRankDynamicShortConvolution(nn.Module):
    """Low-rank dynamic short convolution with its static (bias) filter.

    forward(x, pre_z): x [B, T, d_model] is convolved, pre_z [B, T, d_model] (the
    pre-norm activations) produces the rank-R mixing coefficients z.
    """

    def __init__(self, d_model: int, R: int, W: int):
        super().__init__()
        _check_rank(R)
        self.d_model, self.R, self.W = d_model, R, W
        self.proj_in = nn.Linear(d_model, R, bias=False)
        self.proj_out = nn.Parameter(torch.zeros(R, W * d_model))
        self.proj_out_bias = nn.Parameter(torch.empty(W, d_model))
        nn.init.uniform_(self.proj_out_bias, -1.0 / math.sqrt(W), +1.0 / math.sqrt(W))

    def forward(self, x: torch.Tensor, pre_z: torch.Tensor) -> torch.Tensor:
        z = self.proj_in(pre_z)
        return lowrank_dynamic_convolution(
            x=x.contiguous(),
            z=z.contiguous(),
            U=self.proj_out,
            static_w=self.proj_out_bias,
            residual=True,
        )


class QKVLowRankDynamicShortConvolution(nn.Module):
    """The query, key and value convolutions of one attention layer.

    Parameters are those of three ``LowRankDynamicShortConvolution`` modules
    (``q``, ``k``, ``v``).  The three proj_in GEMMs run as one over the stacked
    weights, and the three convolutions as one grouped launch per direction
    (``lowrank_dynamic_convolution_grouped``), with one all-reduce of the stacked
    dU / static_w gradients under ``data_parallel()``.

    ``forward_fused(qkv, pre_z)`` takes the fused projection output [B, T, 3*d_model]
    as it comes out of the QKV GEMM and returns the three results in the same
    layout, with no split or copy.  ``forward(q, k, v, pre_z)`` takes the three
    tensors (concatenated once, as the reference's ``.contiguous()`` calls copy
    them) and returns three [B, T, d_model] views.
    """

    def __init__(self, d_model: int, R: int, W: int):
        super().__init__()
        self.q = LowRankDynamicShortConvolution(d_model, R, W)
        self.k = LowRankDynamicShortConvolution(d_model, R, W)
        self.v = LowRankDynamicShortConvolution(d_model, R, W)

    def forward_fused(self, qkv: torch.Tensor, pre_z: torch.Tensor) -> torch.Tensor:
        mods = (self.q, self.k, self.v)
        w_in = torch.cat([m.proj_in.weight for m in mods], dim=0)  # [3R, d_model]
        z_all = torch.nn.functional.linear(pre_z, w_in)  # [B, T, 3R]
        U = torch.stack([m.proj_out for m in mods])  # [3, R, W*d_model]
        sw = torch.stack([m.proj_out_bias for m in mods])  # [3, W, d_model]
        return lowrank_dynamic_convolution_grouped(qkv.contiguous(), z_all.contiguous(), U, sw, residual=True)

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, pre_z: torch.Tensor):
        y = self.forward_fused(torch.cat([q, k, v], dim=-1), pre_z)
        return y.split(self.q.d_model, dim=-1)
