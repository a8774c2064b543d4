"""ctypes binding of libdynconv.so (the C ABI declared in include/dynconv.h).

The shared library is built in-tree (``python -m dynamic_conv1d_b200.build``) and
loaded from this directory.  There is no fallback: if the library is missing or
cannot be loaded, every op raises.
"""
from __future__ import annotations

import ctypes
import functools
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libdynconv.so")

DTYPE_BF16 = 0
DTYPE_F32 = 1
_TORCH_DTYPES = {torch.bfloat16: DTYPE_BF16, torch.float32: DTYPE_F32}

_c_i64 = ctypes.c_int64
_c_int = ctypes.c_int
_c_vp = ctypes.c_void_p
_c_size = ctypes.c_size_t

_SIGNATURES = {
    "dynconv_abi_version": (_c_int, []),
    "dynconv_status_string": (ctypes.c_char_p, [_c_int]),
    "dynconv_last_error": (ctypes.c_char_p, []),
    "dynconv_check_device": (_c_int, [_c_vp]),
    "dynconv_launch_count": (ctypes.c_uint64, []),
    "dynconv_hw_fwd": (_c_int, [_c_vp] * 4 + [_c_i64] * 5 + [_c_int, _c_int, _c_vp]),
    "dynconv_hw_bwd_workspace_bytes": (_c_size, [_c_i64] * 5 + [_c_int, _c_int]),
    "dynconv_hw_bwd": (_c_int, [_c_vp] * 8 + [_c_vp, _c_size] + [_c_i64] * 5 + [_c_int, _c_int, _c_vp]),
    "dynconv_lr_fwd_workspace_bytes": (_c_size, [_c_i64] * 5 + [_c_int, _c_int]),
    "dynconv_lr_fwd": (_c_int, [_c_vp] * 5 + [_c_vp, _c_size] + [_c_i64] * 5 + [_c_int, _c_int, _c_vp]),
    "dynconv_lr_fwd_noalloc": (_c_int, [_c_vp] * 5 + [_c_i64] * 5 + [_c_int, _c_int, _c_vp]),
    "dynconv_lr_bwd_workspace_bytes": (_c_size, [_c_i64] * 5 + [_c_int, _c_int]),
    "dynconv_lr_bwd": (_c_int, [_c_vp] * 10 + [_c_vp, _c_size] + [_c_i64] * 5 + [_c_int, _c_int, _c_vp]),
    "dynconv_lr_fwd_grouped_workspace_bytes": (_c_size, [_c_i64] * 6 + [_c_int, _c_int]),
    "dynconv_lr_fwd_grouped": (_c_int, [_c_vp] * 5 + [_c_vp, _c_size] + [_c_i64] * 6 + [_c_int, _c_int, _c_vp]),
    "dynconv_lr_bwd_grouped_workspace_bytes": (_c_size, [_c_i64] * 6 + [_c_int, _c_int]),
    "dynconv_lr_bwd_grouped": (_c_int, [_c_vp] * 10 + [_c_vp, _c_size] + [_c_i64] * 6 + [_c_int, _c_int, _c_vp, _c_vp]),
    "dynconv_comm_blob_bytes": (_c_size, []),
    "dynconv_comm_create": (_c_int, [_c_int, _c_int, _c_i64, ctypes.POINTER(_c_vp), _c_vp]),
    "dynconv_comm_connect": (_c_int, [_c_vp, _c_vp]),
    "dynconv_comm_destroy": (_c_int, [_c_vp]),
    "dynconv_lr_bwd_grouped_dp": (_c_int, [_c_vp] * 10 + [_c_vp, _c_size] + [_c_i64] * 6
                                  + [_c_int, _c_int, _c_vp, _c_vp, _c_vp]),
    "dynconv_cast_f32": (_c_int, [_c_vp, _c_vp, _c_i64, _c_int, _c_vp]),
    "dynconv_umma_selftest": (_c_int, [_c_vp, _c_vp, _c_vp] + [_c_int] * 12 + [_c_vp]),
    "dynconv_wait_selftest": (_c_int, [ctypes.c_uint64, _c_vp, _c_vp]),
}

EXPORTED_SYMBOLS = tuple(_SIGNATURES)

_lock = threading.Lock()
_lib = None


class DynconvError(RuntimeError):
    """A libdynconv entry point returned a non-zero status."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def load() -> ctypes.CDLL:
    """Load libdynconv.so (once) and declare its prototypes."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m dynamic_conv1d_b200.build` "
                    "(there is no CPU or non-CUDA fallback)"
                )
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            if lib.dynconv_abi_version() != 1:
                raise RuntimeError("libdynconv ABI version mismatch")
            _lib = lib
    return _lib


def check(status: int) -> None:
    if status != 0:
        lib = load()
        msg = lib.dynconv_last_error().decode(errors="replace")
        kind = lib.dynconv_status_string(status).decode()
        raise DynconvError(status, f"libdynconv: {kind}: {msg}")


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _TORCH_DTYPES[dtype]
    except KeyError:
        raise TypeError(f"dynamic convolution supports bfloat16 and float32 tensors, got {dtype}") from None


def on_device(fn):
    """Runs an autograd forward/backward with its first tensor's device current:
    the library launches on the current device, the stream comes from the tensor."""

    @functools.wraps(fn)
    def wrapper(ctx, first, *args):
        with torch.cuda.device(first.device):
            return fn(ctx, first, *args)

    return wrapper


def ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def check_device(t: torch.Tensor) -> None:
    """Synchronise the current stream and raise if a device-side bounded wait gave up."""
    check(load().dynconv_check_device(stream_of(t)))


_sync_checks = os.environ.get("DYNCONV_SYNC_CHECK", "0") not in ("", "0")


def set_sync_checks(enabled: bool) -> None:
    """Debug mode (also DYNCONV_SYNC_CHECK=1 in the environment): every forward and
    backward call synchronises its stream and raises DynconvError(DYNCONV_ERR_TIMEOUT)
    at the call whose kernel gave up a bounded wait.  Off by default: the normal path
    never synchronises, and a timed-out kernel is reported by the next check_device()."""
    global _sync_checks
    _sync_checks = bool(enabled)


def after_call(t: torch.Tensor) -> None:
    """Called by the ops after their launches; checks the device only in debug mode
    (and never while the stream is being captured into a CUDA graph)."""
    if _sync_checks and not torch.cuda.is_current_stream_capturing():
        check_device(t)
