"""CPU: the C-ABI library loads, exports every entry point that include/dynconv.h
declares, and rejects bad arguments before touching the GPU.  No kernel runs here."""
from __future__ import annotations

import ctypes
import os
import re

import pytest
import torch

from conftest import ROOT
from dynamic_conv1d_b200 import _lib

HEADER = os.path.join(ROOT, "include", "dynconv.h")


def _declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(dynconv_[a-z0-9_]+)\s*\(", src)))


def test_library_present_and_loads():
    assert os.path.exists(_lib.LIB_PATH), "build with python -m dynamic_conv1d_b200.build"
    lib = _lib.load()
    assert lib.dynconv_abi_version() == 1


def test_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    declared = _declared_functions()
    assert len(declared) >= 12
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in dynconv.h but not exported"
    # and the Python binding covers the same set
    assert set(declared) == set(_lib.EXPORTED_SYMBOLS)


def test_status_strings():
    lib = _lib.load()
    for code in range(0, 8):
        assert lib.dynconv_status_string(code)
    assert lib.dynconv_status_string(0) == b"ok"


def _hw_fwd(**kw):
    lib = _lib.load()
    a = dict(x=None, w=None, sw=None, y=None, B=1, T=4, D=16, H=16, W=4, dtype=0, residual=0)
    a.update(kw)
    return lib.dynconv_hw_fwd(a["x"], a["w"], a["sw"], a["y"], a["B"], a["T"], a["D"], a["H"], a["W"],
                              a["dtype"], a["residual"], None)


def test_validation_without_gpu():
    lib = _lib.load()
    assert _hw_fwd(W=9) == 3  # unsupported W
    assert _hw_fwd(D=16, H=3) == 1  # D % H
    assert _hw_fwd(D=24, H=2) == 3  # head size 12 not a power of two
    assert _hw_fwd(dtype=7) == 3
    assert _hw_fwd(B=0) == 0  # empty batch is a no-op
    assert _hw_fwd() == 7  # null tensors
    assert b"null" in lib.dynconv_last_error()
    # lowrank: R_kernel > 64 and missing accumulator
    st = lib.dynconv_lr_fwd(None, None, None, None, None, None, 0, 1, 4, 16, 65, 4, 0, 0, None)
    assert st == 3
    st = lib.dynconv_lr_bwd(*([None] * 10), None, 0, 1, 4, 16, 15, 4, 0, 0, None)
    assert st == 7


def test_workspace_sizes():
    lib = _lib.load()
    assert lib.dynconv_hw_bwd_workspace_bytes(4, 4096, 2048, 64, 4, 0, 0) == 0
    n = lib.dynconv_hw_bwd_workspace_bytes(4, 4096, 2048, 64, 4, 0, 1)
    assert n > 0 and n % 256 == 0
    # partial rows stay a small fraction of the streamed bytes (cfg2: ~360 MB)
    assert n < 8 << 20
    m = lib.dynconv_lr_bwd_workspace_bytes(4, 4096, 2048, 15, 4, 0, 1)
    assert m > 0


def test_api_asserts_like_reference():
    from dynamic_conv1d_b200 import headwise_dynamic_convolution, lowrank_dynamic_convolution

    x = torch.zeros(1, 4, 8)
    w = torch.zeros(1, 4, 8, 2)
    with pytest.raises(AssertionError):
        headwise_dynamic_convolution(x, w)  # not CUDA (headwise.py:332)
    z = torch.zeros(1, 4, 3)
    U = torch.zeros(3, 16)
    with pytest.raises(AssertionError):
        lowrank_dynamic_convolution(x, z, U)  # not CUDA (lowrank.py:328)


def test_dtype_codes():
    assert _lib.dtype_code(torch.bfloat16) == 0
    assert _lib.dtype_code(torch.float32) == 1
    with pytest.raises(TypeError):
        _lib.dtype_code(torch.float16)
