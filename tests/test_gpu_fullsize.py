"""GPU parity at the BASELINE.json benchmark shapes (configs[1..4]) against the CPU
oracle on the same bf16 values: relative L2 <= 1e-2 (y) and <= 2e-2 (gradients).
configs[4] (the data-parallel scale-out, 8 rows of T=8192, D=4096 per GPU at 8
GPUs) is checked on one full row: the same tiles, rank 32 and channel blocks per
tile as every rank runs, at a size the numpy oracle finishes in seconds.

At these sizes every CTA of the persistent kernels walks many tiles, the dz
reduction crosses all 16 channel-block CTAs of a tile, and the dU / dstatic_w
partials of all groups are summed -- paths the small shapes do not reach."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from conftest import rel_l2
from dynamic_conv1d_b200 import headwise_dynamic_convolution, lowrank_dynamic_convolution

pytestmark = pytest.mark.gpu

CONFIGS = {
    "cfg2_headwise_hs32": dict(kind="headwise", B=4, T=4096, D=2048, H=64, W=4),
    "cfg3_headwise_hs1": dict(kind="headwise", B=4, T=4096, D=2048, H=2048, W=4),
    "cfg4_lowrank_r15_static": dict(kind="lowrank", B=4, T=4096, D=2048, R=15, W=4),
    "cfg5_lowrank_r31_static_row": dict(kind="lowrank", B=1, T=8192, D=4096, R=31, W=4),
}


@pytest.mark.parametrize("name", list(CONFIGS))
def test_full_size(name, cuda_device):
    c = CONFIGS[name]
    B, T, D, W = c["B"], c["T"], c["D"], c["W"]
    g = torch.Generator().manual_seed(11)
    bf = torch.bfloat16

    def rnd(*shape, scale=1.0):
        return (torch.randn(*shape, generator=g) * scale).to(bf)

    x, dy = rnd(B, T, D), rnd(B, T, D)
    if c["kind"] == "headwise":
        w = rnd(B, T, c["H"], W)
        sw = rnd(W, D)
        cpu = [x, w, sw]
        fn = headwise_dynamic_convolution
    else:
        R = c["R"]
        z = rnd(B, T, R)
        U = rnd(R, W * D, scale=1.0 / np.sqrt(R))
        sw = (torch.rand(W, D, generator=g) - 0.5).to(bf)
        cpu = [x, z, U, sw]
        fn = lowrank_dynamic_convolution
    leaves = [t.to(cuda_device).requires_grad_() for t in cpu]
    y = fn(*leaves, residual=True)
    y.backward(dy.to(cuda_device))
    torch.cuda.synchronize()
    f = [t.float().numpy() for t in cpu]
    if c["kind"] == "headwise":
        ry = oracle.headwise_fwd(f[0], f[1], f[2], True)
        grads = oracle.headwise_bwd(f[0], f[1], f[2], dy.float().numpy(), True)
    else:
        ry = oracle.lowrank_fwd(f[0], f[1], f[2], f[3], True)
        grads = oracle.lowrank_bwd(f[0], f[1], f[2], f[3], dy.float().numpy(), True)
    e = rel_l2(y.detach().float().cpu().numpy(), ry)
    assert e <= 1e-2, f"{name} y rel-L2 {e:.3e}"
    for leaf, ref, nm in zip(leaves, grads, ["dx", "d1", "d2", "d3"]):
        e = rel_l2(leaf.grad.float().cpu().numpy(), ref)
        assert e <= 2e-2, f"{name} {nm} rel-L2 {e:.3e}"
