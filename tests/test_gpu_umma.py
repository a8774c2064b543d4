"""GPU: tcgen05.mma descriptor encodings of the lowrank tensor-core kernels.

Each case stages bf16 operands into the exact no-swizzle shared-memory layouts
that one MMA of the lowrank kernels uses (K-major or MN-major, SBO/LBO strides,
row-shifted B) and compares D = A @ B with a float32 torch matmul."""
from __future__ import annotations

import ctypes
import zlib

import pytest
import torch

from dynamic_conv1d_b200 import _lib

pytestmark = pytest.mark.gpu

# name: (M, N, K, Nb, a_major, a_sbo, a_lbo, b_major, b_sbo, b_lbo, b_row_offset)
CASES = {
    # forward / dx weight generation: A = U_w^T [128 ch x R] K-major, B = z [tok x R] K-major
    "fwd_R16": (128, 64, 16, 64, 0, 256, 128, 0, 128, 64 * 16, 0),
    "fwd_R32": (128, 64, 32, 64, 0, 512, 128, 0, 128, 64 * 16, 0),
    # dx: the same z buffer read from row w (shifted start address)
    "dx_shift1": (128, 64, 16, 72, 0, 256, 128, 0, 128, 72 * 16, 1),
    "dx_shift3": (128, 64, 16, 72, 0, 256, 128, 0, 128, 72 * 16, 3),
    # dU: A = P^T [128 ch x 64 tok] K-major, B = z [64 tok x R] MN-major (the z buffer)
    "dU_R16": (128, 16, 64, 16, 0, 1024, 128, 1, 72 * 16, 128, 0),
    "dU_R32": (128, 32, 64, 32, 0, 1024, 128, 1, 72 * 16, 128, 0),
    # dz: A = P [64 tok x 128 ch] MN-major (M = 64), B = U [128 ch x R] MN-major
    "dz_R16": (64, 16, 128, 16, 1, 128, 1024, 1, 128, 256, 0),
    "dz_R32": (64, 32, 128, 32, 1, 128, 1024, 1, 128, 512, 0),
    # wide N, two K steps
    "wide": (128, 256, 32, 256, 0, 512, 128, 0, 512, 128, 0),
    # A operand in tensor memory (a_major = 2): weight MMAs (A = U) and the dU MMA (A = P^T)
    "tmemA_fwd_R16": (128, 64, 16, 64, 2, 0, 0, 0, 128, 64 * 16, 0),
    "tmemA_fwd_R32": (128, 64, 32, 64, 2, 0, 0, 0, 128, 64 * 16, 0),
    "tmemA_dx_shift2": (128, 32, 16, 72, 2, 0, 0, 0, 128, 72 * 16, 2),
    "tmemA_dU_R16": (128, 16, 64, 16, 2, 0, 0, 1, 72 * 16, 128, 0),
    "tmemA_dU_R32": (128, 32, 64, 32, 2, 0, 0, 1, 72 * 16, 128, 0),
    # backward, per 16-step quarter: weight MMA (N = 16, z rows from 16i + w) and dU MMA (K = 16)
    "tmemA_q_shift3": (128, 16, 16, 72, 2, 0, 0, 0, 128, 72 * 16, 3),
    "tmemA_q_shift51": (128, 16, 32, 72, 2, 0, 0, 0, 128, 72 * 16, 51),
    "tmemA_q_dU_R16": (128, 16, 16, 16, 2, 0, 0, 1, 72 * 16, 128, 0),
    "tmemA_q_dU_R32": (128, 32, 16, 32, 2, 0, 0, 1, 72 * 16, 128, 0),
    # 128-byte-swizzled MN-major A (a_major = 3): a 16-row block of a SWIZZLE_128B TMA
    # tile, 64-channel atoms LBO apart -- the backward's transposing MMA (B = identity)
    "sw128_transpose": (128, 16, 16, 16, 3, 1024, 2048, 0, 128, 256, 0),
    "sw128_K32": (128, 32, 32, 32, 3, 1024, 4096, 0, 128, 512, 0),
    "sw128_M64": (64, 16, 16, 16, 3, 1024, 2048, 0, 128, 256, 0),
    # forward weight MMA: A = U^T MN-major (16-byte rows of 8 channels; 8-channel groups
    # RKP/8 x 128 B apart, 8-rank groups 128 B apart), B = z K-major
    "fwd_mnA_R16": (128, 64, 16, 64, 1, 256, 128, 0, 128, 64 * 16, 0),
    "fwd_mnA_R32": (128, 64, 32, 64, 1, 512, 128, 0, 128, 64 * 16, 0),
    "fwd_mnA_R64": (128, 64, 64, 64, 1, 1024, 128, 0, 128, 64 * 16, 0),
    # time-major backward (M = 128 timesteps): weight MMA, A = z rows t+w (K-major, rows
    # 16 B apart, 8-rank chunks 136 rows apart), B = U tap w (MN-major, N = 32 channels)
    "tm_w_R16": (128, 32, 16, 32, 0, 128, 136 * 16, 1, 256, 128, 0, 0),
    "tm_w_R16_shift3": (128, 32, 16, 32, 0, 128, 136 * 16, 1, 256, 128, 0, 3),
    "tm_w_R32_shift2": (128, 32, 32, 32, 0, 128, 136 * 16, 1, 512, 128, 0, 2),
    # dz MMA: A = P [t][(tap, ch)] K-major (8-step groups 2048 B apart), B = U K-major
    "tm_dz_R16": (128, 16, 32, 16, 0, 2048, 128, 0, 128, 256, 0),
    "tm_dz_R32": (128, 32, 32, 32, 0, 2048, 128, 0, 128, 512, 0),
    # dU MMA: A = the same P buffer read MN-major (M = 4 taps x 32 channels), B = z MN-major
    "tm_dU_R16": (128, 16, 128, 16, 1, 128, 2048, 1, 136 * 16, 128, 0),
    "tm_dU_R32": (128, 32, 128, 32, 1, 128, 2048, 1, 136 * 16, 128, 0),
}


@pytest.mark.parametrize("name", list(CASES))
def test_umma_layout(name, cuda_device):
    M, N, K, Nb, am, asbo, albo, bm, bsbo, blbo, off, *rest = CASES[name]
    a_off = rest[0] if rest else 0
    g = torch.Generator(device="cuda").manual_seed(zlib.crc32(name.encode()))
    A = torch.randn(M + a_off, K, device="cuda", generator=g).to(torch.bfloat16)
    B = torch.randn(K, Nb, device="cuda", generator=g).to(torch.bfloat16)
    D = torch.full((M, N), float("nan"), device="cuda", dtype=torch.float32)
    lib = _lib.load()
    st = lib.dynconv_umma_selftest(
        ctypes.c_void_p(A.data_ptr()), ctypes.c_void_p(B.data_ptr()), ctypes.c_void_p(D.data_ptr()),
        M, N, K, Nb, am, asbo, albo, bm, bsbo, blbo, off, a_off, _lib.stream_of(A),
    )
    _lib.check(st)
    _lib.check_device(A)
    ref = A.float()[a_off:a_off + M] @ B.float()[:, off:off + N]
    torch.testing.assert_close(D, ref, atol=1e-3, rtol=1e-3)


def test_transpose_is_exact(cuda_device):
    """The identity MMA used to transpose dy/x tiles returns every bf16 value exactly."""
    M, N, K = 128, 16, 16
    g = torch.Generator(device="cuda").manual_seed(5)
    A = (torch.randn(M, K, device="cuda", generator=g) * 1e3).to(torch.bfloat16)
    B = torch.eye(K, N, device="cuda").to(torch.bfloat16)
    D = torch.full((M, N), float("nan"), device="cuda", dtype=torch.float32)
    lib = _lib.load()
    _lib.check(lib.dynconv_umma_selftest(
        ctypes.c_void_p(A.data_ptr()), ctypes.c_void_p(B.data_ptr()), ctypes.c_void_p(D.data_ptr()),
        M, N, K, K, 3, 1024, 2048, 0, 128, 256, 0, 0, _lib.stream_of(A),
    ))
    _lib.check_device(A)
    assert torch.equal(D, A.float())
