"""GPU: the bounded-wait (fault-containment) path.

A one-CTA kernel waits on an mbarrier that nothing ever arrives on, through the
same out-of-line bounded-wait code the tensor-core kernels use, with a 2 ms
limit.  The wait gives up, the kernel returns, and the host sees
DYNCONV_ERR_TIMEOUT from dynconv_check_device(), from the next op call (which
reads the pinned host-visible error word), and from the op in debug mode -- with
the CUDA context still usable: the next op runs and matches the oracle.
No GPU fault, trap or hang is involved: the kernel simply exits early."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import oracle
from dynamic_conv1d_b200 import DynconvError, _lib, check_device, lowrank_dynamic_convolution, set_sync_checks

pytestmark = pytest.mark.gpu

DYNCONV_ERR_TIMEOUT = 5
DYNCONV_ERR_ARGUMENT = 7
LIMIT_NS = 2_000_000  # 2 ms


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _run_wait(out):
    lib = _lib.load()
    _lib.check(lib.dynconv_wait_selftest(ctypes.c_uint64(LIMIT_NS), ctypes.c_void_p(out.data_ptr()), _stream()))


def _small_lowrank():
    g = torch.Generator().manual_seed(5)
    B, T, D, R, W = 1, 200, 256, 15, 4
    x = torch.randn(B, T, D, generator=g).to(torch.bfloat16)
    z = (torch.randn(B, T, R, generator=g) * 0.3).to(torch.bfloat16)
    U = (torch.randn(R, W * D, generator=g) * 0.25).to(torch.bfloat16)
    sw = (torch.randn(W, D, generator=g) * 0.3).to(torch.bfloat16)
    return x, z, U, sw


def _check_small_lowrank():
    x, z, U, sw = _small_lowrank()
    y = lowrank_dynamic_convolution(*(t.cuda() for t in (x, z, U, sw)), residual=True)
    ref = oracle.lowrank_fwd(*(t.float().numpy() for t in (x, z, U, sw)), True)
    yd = y.float().cpu().numpy().astype(np.float64)
    rel = np.linalg.norm(yd - ref) / np.linalg.norm(ref)
    assert rel < 1e-2, rel


def test_wait_gives_up_and_reports_timeout():
    torch.cuda.synchronize()
    check_device(torch.empty(1, device="cuda"))  # start from a clean error word
    out = torch.full((1,), 7, dtype=torch.int32, device="cuda")
    _run_wait(out)
    lib = _lib.load()
    status = lib.dynconv_check_device(_stream())
    assert status == DYNCONV_ERR_TIMEOUT, (status, lib.dynconv_last_error())
    assert b"self-test" in lib.dynconv_last_error()
    assert int(out.item()) == 0  # the wait returned "gave up"
    # the word was cleared by the read: the next check is clean
    assert lib.dynconv_check_device(_stream()) == 0
    # the context is intact: a real op runs and matches the oracle
    _check_small_lowrank()
    assert lib.dynconv_check_device(_stream()) == 0


def test_next_call_reports_timeout_without_check_device():
    """A kernel that gave up a wait is reported by the next op call itself (the host
    reads the pinned error word, no synchronisation), once; then calls run normally."""
    torch.cuda.synchronize()
    check_device(torch.empty(1, device="cuda"))  # start clean
    x, z, U, sw = (t.cuda() for t in _small_lowrank())
    lowrank_dynamic_convolution(x, z, U, sw, residual=True)  # this device's error word is wired
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    _run_wait(out)
    torch.cuda.synchronize()  # the self-test kernel has finished; no check_device
    with pytest.raises(DynconvError) as ei:
        lowrank_dynamic_convolution(x, z, U, sw, residual=True)
    assert ei.value.status == DYNCONV_ERR_TIMEOUT
    assert "earlier" in str(ei.value)
    # reported once, device words cleared with it: the next call runs and check_device is clean
    _check_small_lowrank()
    check_device(out)


def test_check_device_raises():
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    _run_wait(out)
    with pytest.raises(DynconvError) as ei:
        check_device(out)
    assert ei.value.status == DYNCONV_ERR_TIMEOUT
    check_device(out)  # cleared


def test_sync_check_mode_raises_at_the_call():
    """In debug mode the first op after the timed-out kernel raises at its own call."""
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    x, z, U, sw = (t.cuda() for t in _small_lowrank())
    set_sync_checks(True)
    try:
        _run_wait(out)
        with pytest.raises(DynconvError) as ei:
            lowrank_dynamic_convolution(x, z, U, sw, residual=True)
        assert ei.value.status == DYNCONV_ERR_TIMEOUT
        lowrank_dynamic_convolution(x, z, U, sw, residual=True)  # clean again
    finally:
        set_sync_checks(False)


def test_limit_argument_checked():
    lib = _lib.load()
    assert lib.dynconv_wait_selftest(ctypes.c_uint64(0), None, _stream()) == DYNCONV_ERR_ARGUMENT
    assert lib.dynconv_wait_selftest(ctypes.c_uint64(10**9), None, _stream()) == DYNCONV_ERR_ARGUMENT
