"""dynconv_lr_fwd_noalloc (scratch in a static device array, no workspace argument)
against dynconv_lr_fwd (caller workspace), both called through the C ABI.

The file name sorts last so that pytest collects it after every other test; it
also passes when run alone.  Two calls in a row with different inputs and sizes
show that the shared scratch is rewritten by each call."""
from __future__ import annotations

import pytest
import torch

from dynamic_conv1d_b200 import _lib

pytestmark = pytest.mark.gpu

BF16_TOL = dict(atol=1e-2, rtol=1e-2)


def _inputs(B, T, D, R, W, seed, dev):
    g = torch.Generator().manual_seed(seed)
    bf = torch.bfloat16
    x = torch.randn(B, T, D, generator=g).to(bf)
    z = torch.randn(B, T, R, generator=g).to(bf)
    U = (torch.randn(R, W * D, generator=g) / R**0.5).to(bf)
    sw = (torch.rand(W, D, generator=g) - 0.5).to(bf)
    return [t.to(dev) for t in (x, z, U, sw)]


def _lr_fwd_workspace(lib, x, z, U, sw, residual):
    B, T, D = x.shape
    R = z.shape[-1]
    W = U.shape[-1] // D
    code = _lib.dtype_code(x.dtype)
    y = torch.empty_like(x)
    nbytes = lib.dynconv_lr_fwd_workspace_bytes(B, T, D, R, W, code, int(sw is not None))
    ws = torch.empty(max(int(nbytes), 1), device=x.device, dtype=torch.uint8)
    _lib.check(lib.dynconv_lr_fwd(_lib.ptr(x), _lib.ptr(z), _lib.ptr(U), _lib.ptr(sw), _lib.ptr(y), _lib.ptr(ws),
                                  ws.numel(), B, T, D, R, W, code, int(residual), _lib.stream_of(x)))
    return y


def _lr_fwd_noalloc(lib, x, z, U, sw, residual):
    B, T, D = x.shape
    R = z.shape[-1]
    W = U.shape[-1] // D
    y = torch.empty_like(x)
    _lib.check(lib.dynconv_lr_fwd_noalloc(_lib.ptr(x), _lib.ptr(z), _lib.ptr(U), _lib.ptr(sw), _lib.ptr(y), B, T, D,
                                          R, W, _lib.dtype_code(x.dtype), int(residual), _lib.stream_of(x)))
    return y


def test_noalloc_matches_workspace_entry_point(cuda_device):
    lib = _lib.load()
    cases = [
        # (B, T, D, R, W, static, residual, seed)
        (2, 700, 256, 15, 4, True, True, 1),
        (3, 129, 512, 31, 3, True, False, 2),
    ]
    for B, T, D, R, W, static, residual, seed in cases:
        x, z, U, sw = _inputs(B, T, D, R, W, seed, cuda_device)
        sw = sw if static else None
        want = _lr_fwd_workspace(lib, x, z, U, sw, residual)
        got = _lr_fwd_noalloc(lib, x, z, U, sw, residual)
        torch.cuda.synchronize()
        _lib.check_device(x)
        torch.testing.assert_close(got, want, **BF16_TOL)


def test_noalloc_rejects_sizes_beyond_scratch(cuda_device):
    lib = _lib.load()
    # B*T*16 bf16 = 16 MiB of packed z, above the fixed 8 MiB scratch; rejected
    # before any tensor is touched.
    status = lib.dynconv_lr_fwd_noalloc(None, None, None, None, None, 8, 65536, 256, 15, 4,
                                        _lib.dtype_code(torch.bfloat16), 1, None)
    assert status == 6  # DYNCONV_ERR_WORKSPACE
    assert "scratch" in lib.dynconv_last_error().decode()
