"""GPU: the grouped (Q/K/V) lowrank convolution -- G convolutions in one launch
per direction -- against G separate oracle calls, one per channel group.

Tolerances as everywhere: relative L2 <= 1e-2 for y, <= 2e-2 for gradients."""
from __future__ import annotations

import zlib

import numpy as np
import pytest
import torch

import oracle
from conftest import rel_l2
from dynamic_conv1d_b200 import _lib, lowrank_dynamic_convolution_grouped
from dynamic_conv1d_b200.lowrank import _LowrankGroupedFn

pytestmark = pytest.mark.gpu

# G, B, T, D, R, W, static, residual
CASES = [
    (3, 2, 300, 256, 15, 4, True, True),
    (3, 1, 4096, 2048, 15, 4, True, True),   # cfg4 channels: 48 channel blocks, many tiles per CTA
    (2, 2, 1000, 512, 31, 3, True, False),   # R_kernel = 32
    (3, 2, 200, 128, 16, 2, False, True),    # no static rank
    (4, 1, 130, 384, 7, 1, True, True),      # W = 1, ragged T
]


def _inputs(case, dtype=torch.bfloat16):
    G, B, T, D, R, W, st, _ = case
    rng = np.random.default_rng(zlib.crc32(repr(case).encode()))

    def rnd(*shape, scale=1.0):
        return torch.from_numpy((rng.standard_normal(shape) * scale).astype(np.float32)).to(dtype)

    x, dy = rnd(B, T, G * D), rnd(B, T, G * D)
    z = rnd(B, T, G * R, scale=0.5)
    U = rnd(G, R, W * D, scale=1.0 / np.sqrt(R))
    sw = rnd(G, W, D, scale=0.3) if st else None
    return x, z, U, sw, dy


def _oracle_groups(case, x, z, U, sw, dy):
    G, B, T, D, R, W, st, res = case
    f = lambda t: t.float().numpy()
    ys, dxs, dzs, dUs, dsws = [], [], [], [], []
    for g in range(G):
        xg, zg = f(x)[..., g * D:(g + 1) * D], f(z)[..., g * R:(g + 1) * R]
        swg = f(sw[g]) if st else None
        ys.append(oracle.lowrank_fwd(xg, zg, f(U[g]), swg, res))
        dx, dz, dU, dsw = oracle.lowrank_bwd(xg, zg, f(U[g]), swg, f(dy)[..., g * D:(g + 1) * D], res)
        dxs.append(dx), dzs.append(dz), dUs.append(dU), dsws.append(dsw)
    out = {"y": np.concatenate(ys, -1), "dx": np.concatenate(dxs, -1), "dz": np.concatenate(dzs, -1),
           "dU": np.stack(dUs)}
    if st:
        out["dsw"] = np.stack(dsws)
    return out


def _run(case, cuda_device, dtype=torch.bfloat16):
    x, z, U, sw, dy = _inputs(case, dtype)
    leaves = [t.to(cuda_device).requires_grad_() for t in (x, z, U) + ((sw,) if sw is not None else ())]
    y = lowrank_dynamic_convolution_grouped(*leaves[:3], leaves[3] if sw is not None else None, residual=case[7])
    y.backward(dy.to(cuda_device))
    torch.cuda.synchronize()
    got = {"y": y, "dx": leaves[0].grad, "dz": leaves[1].grad, "dU": leaves[2].grad}
    if sw is not None:
        got["dsw"] = leaves[3].grad
    return got, _oracle_groups(case, x, z, U, sw, dy)


@pytest.mark.parametrize("case", CASES, ids=lambda c: "-".join(str(v) for v in c))
def test_grouped_matches_per_group_oracle(case, cuda_device):
    got, ref = _run(case, cuda_device)
    for k, r in ref.items():
        g = got[k].detach().float().cpu().numpy()
        assert g.shape == r.shape, (k, g.shape, r.shape)
        e = rel_l2(g, r)
        assert e <= (1e-2 if k == "y" else 2e-2), f"{k} rel-L2 {e:.3e}"


def test_grouped_is_one_launch_per_direction(cuda_device):
    """z packing + the forward kernel, then the backward kernel alone (it reads the z
    the forward packed): three launches for all three groups (three separate calls
    launch nine)."""
    case = (3, 2, 256, 256, 15, 4, True, True)
    x, z, U, sw, dy = (t.to(cuda_device) for t in _inputs(case))
    leaves = [t.requires_grad_() for t in (x, z, U, sw)]
    lib = _lib.load()
    torch.cuda.synchronize()
    n0 = lib.dynconv_launch_count()
    y = _LowrankGroupedFn.apply(*leaves, True)
    n1 = lib.dynconv_launch_count()
    y.backward(dy)
    torch.cuda.synchronize()
    n2 = lib.dynconv_launch_count()
    assert (n1 - n0, n2 - n1) == (2, 1)


def test_grouped_matches_separate_calls_bitwise(cuda_device):
    """Each group's results equal the single op's on that group's slice, bit for bit
    (same kernels, same reduction order)."""
    from dynamic_conv1d_b200 import lowrank_dynamic_convolution

    case = (3, 2, 500, 256, 15, 4, True, True)
    G, B, T, D, R, W = case[:6]
    x, z, U, sw, dy = (t.to(cuda_device) for t in _inputs(case))
    leaves = [t.clone().requires_grad_() for t in (x, z, U, sw)]
    y = lowrank_dynamic_convolution_grouped(*leaves, residual=True)
    y.backward(dy)
    for g in range(G):
        sl = slice(g * D, (g + 1) * D)
        lg = [x[..., sl].contiguous().requires_grad_(), z[..., g * R:(g + 1) * R].contiguous().requires_grad_(),
              U[g].clone().requires_grad_(), sw[g].clone().requires_grad_()]
        yg = lowrank_dynamic_convolution(*lg, residual=True)
        yg.backward(dy[..., sl].contiguous())
        assert torch.equal(y[..., sl], yg)
        assert torch.equal(leaves[0].grad[..., sl], lg[0].grad)
        assert torch.equal(leaves[1].grad[..., g * R:(g + 1) * R], lg[1].grad)
        assert torch.equal(leaves[2].grad[g], lg[2].grad)
        assert torch.equal(leaves[3].grad[g], lg[3].grad)


def test_grouped_fallback_float32(cuda_device):
    """Outside the grouped kernels' envelope (float32 here) the groups run one by one."""
    case = (3, 1, 150, 64, 15, 4, True, True)
    got, ref = _run(case, cuda_device, torch.float32)
    for k, r in ref.items():
        e = rel_l2(got[k].detach().float().cpu().numpy(), r)
        assert e <= 1e-4, f"{k} rel-L2 {e:.3e}"


def test_grouped_unsupported_is_reported(cuda_device):
    """The C ABI refuses G > 1 outside the tensor-core envelope instead of guessing."""
    lib = _lib.load()
    B, T, D, R, W, G = 1, 64, 96, 15, 4, 3  # D % 128 != 0
    x = torch.zeros(B, T, G * D, device=cuda_device, dtype=torch.bfloat16)
    z = torch.zeros(B, T, G * R, device=cuda_device, dtype=torch.bfloat16)
    U = torch.zeros(G, R, W * D, device=cuda_device, dtype=torch.bfloat16)
    y = torch.empty_like(x)
    st = _lib.stream_of(x)
    s = lib.dynconv_lr_fwd_grouped(_lib.ptr(x), _lib.ptr(z), _lib.ptr(U), None, _lib.ptr(y), None, 0,
                                   B, T, D, R, W, G, 0, 1, st)
    assert s == 3 and b"tensor-core path" in lib.dynconv_last_error()  # DYNCONV_ERR_UNSUPPORTED
