"""B200-native dynamic short convolutions (drop-in for OliverSieberling/dynamic-conv1d).

    from dynamic_conv1d_b200 import headwise_dynamic_convolution, lowrank_dynamic_convolution

Both ops are ``torch.autograd.Function``s over libdynconv.so, a C-ABI library of
hand-written sm_100a CUDA kernels (see ``include/dynconv.h``).

Calls never synchronise.  The tensor-core kernels bound every device-side wait
(1.5 s); a wait that gives up makes its kernel return early and sets a device
error word, which ``check_device(t)`` reads (raising ``DynconvError`` with status
DYNCONV_ERR_TIMEOUT).  Call it once per training step (or set DYNCONV_SYNC_CHECK=1
/ ``set_sync_checks(True)`` to check after every call while debugging).
"""
from ._lib import DynconvError, check_device, set_sync_checks
from .headwise import headwise_dynamic_convolution
from .lowrank import lowrank_dynamic_convolution, lowrank_dynamic_convolution_grouped
from .modules import LowRankDynamicShortConvolution, QKVLowRankDynamicShortConvolution
from .parallel import data_parallel, shard_rows
from .sequence_parallel import headwise_dynamic_convolution_sp, lowrank_dynamic_convolution_sp

__all__ = [
    "headwise_dynamic_convolution",
    "lowrank_dynamic_convolution",
    "lowrank_dynamic_convolution_grouped",
    "LowRankDynamicShortConvolution",
    "QKVLowRankDynamicShortConvolution",
    "data_parallel",
    "lowrank_dynamic_convolution_sp",
    "headwise_dynamic_convolution_sp",
    "shard_rows",
    "check_device",
    "set_sync_checks",
    "DynconvError",
]
