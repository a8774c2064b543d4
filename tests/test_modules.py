"""The README modules (reference README.md:57-105): parameters, initialisation and
errors on CPU; forward / backward on a GPU against the oracle, and the grouped
Q/K/V module against three separate modules."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import oracle
from conftest import rel_l2
from dynamic_conv1d_b200 import LowRankDynamicShortConvolution, QKVLowRankDynamicShortConvolution


def test_module_parameters_and_init():
    torch.manual_seed(0)
    m = LowRankDynamicShortConvolution(64, R=15, W=4)
    assert m.proj_in.weight.shape == (15, 64) and m.proj_in.bias is None
    assert m.proj_out.shape == (15, 4 * 64) and torch.count_nonzero(m.proj_out) == 0
    assert m.proj_out_bias.shape == (4, 64)
    assert float(m.proj_out_bias.detach().abs().max()) <= 1.0 / math.sqrt(4)
    with pytest.raises(ValueError):
        LowRankDynamicShortConvolution(64, R=16, W=4)  # R+1 not a power of two


def test_qkv_module_holds_three_modules():
    m = QKVLowRankDynamicShortConvolution(64, R=7, W=3)
    assert sum(p.numel() for p in m.parameters()) == 3 * (7 * 64 + 7 * 3 * 64 + 3 * 64)


@pytest.mark.gpu
def test_module_forward_backward_matches_oracle(cuda_device):
    torch.manual_seed(1)
    B, T, D, R, W = 2, 160, 256, 15, 4
    m = LowRankDynamicShortConvolution(D, R, W).to(cuda_device, torch.bfloat16)
    with torch.no_grad():  # nonzero U so the dynamic part is exercised
        m.proj_out.copy_((torch.randn(R, W * D) * 0.2).to(torch.bfloat16))
    x = torch.randn(B, T, D, device=cuda_device).to(torch.bfloat16).requires_grad_()
    pre = torch.randn(B, T, D, device=cuda_device).to(torch.bfloat16)
    y = m(x, pre)
    dy = torch.randn_like(y)
    y.backward(dy)
    torch.cuda.synchronize()
    z = m.proj_in(pre).detach()
    f = lambda t: t.detach().float().cpu().numpy()
    ry = oracle.lowrank_fwd(f(x), f(z), f(m.proj_out), f(m.proj_out_bias), True)
    rdx, _, rdU, rdsw = oracle.lowrank_bwd(f(x), f(z), f(m.proj_out), f(m.proj_out_bias), f(dy), True)
    assert rel_l2(f(y), ry) <= 1e-2
    assert rel_l2(f(x.grad), rdx) <= 2e-2
    assert rel_l2(f(m.proj_out.grad), rdU) <= 2e-2
    assert rel_l2(f(m.proj_out_bias.grad), rdsw) <= 2e-2
    assert m.proj_in.weight.grad is not None and torch.isfinite(m.proj_in.weight.grad.float()).all()


@pytest.mark.gpu
def test_qkv_module_matches_separate_modules(cuda_device):
    torch.manual_seed(2)
    B, T, D, R, W = 2, 96, 128, 15, 4
    qkv = QKVLowRankDynamicShortConvolution(D, R, W).to(cuda_device, torch.bfloat16)
    with torch.no_grad():
        for mm in (qkv.q, qkv.k, qkv.v):
            mm.proj_out.copy_((torch.randn(R, W * D) * 0.2).to(torch.bfloat16))
    q, k, v, pre = (torch.randn(B, T, D, device=cuda_device).to(torch.bfloat16) for _ in range(4))
    outs = qkv(q, k, v, pre)
    for mm, t, o in zip((qkv.q, qkv.k, qkv.v), (q, k, v), outs):
        ref = mm(t, pre)
        assert rel_l2(o.detach().float().cpu().numpy(), ref.detach().float().cpu().numpy()) <= 1e-2
