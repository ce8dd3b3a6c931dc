"""The tensor-core building blocks of the chunked kernels (tcgen05 MMA with
tf32 or bf16 operands from 128-byte swizzled shared memory or tensor memory,
fp32 accumulation in tensor memory) against a float64 host matmul, for every
operand layout the chunked kernels use."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from visionstack_b200 import _lib

pytestmark = pytest.mark.gpu

# mode: (K, N, A MN-major, B MN-major); modes 4-8 read A from tensor memory,
# modes 7-10 take bf16 operands (9-10 with both operands in shared memory)
SHAPES = {0: (128, 64, False, False), 1: (128, 128, False, True), 2: (64, 128, False, True),
          3: (64, 128, True, True), 4: (128, 128, False, False), 5: (64, 64, False, False),
          6: (64, 128, False, True), 7: (128, 128, False, False), 8: (64, 128, False, True),
          9: (128, 64, False, True), 10: (64, 64, True, True)}
BF16_MODES = (7, 8, 9, 10)


def _bf16(x):
    """Round float32 to bf16 (nearest, ties to even) and back."""
    u = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


@pytest.mark.parametrize("mode", sorted(SHAPES))
def test_umma_layouts(mode):
    K, N, a_mn, b_mn = SHAPES[mode]
    rng = np.random.default_rng(mode)
    A = rng.standard_normal((K, 128) if a_mn else (128, K)).astype(np.float32)
    B = rng.standard_normal((N, K) if not b_mn else (K, N)).astype(np.float32)
    Am = A.T if a_mn else A
    Bm = B.T if not b_mn else B
    if mode in BF16_MODES:  # the device rounds the operands to bf16; the products are exact
        Am, Bm = _bf16(Am), _bf16(Bm)
    ref = Am.astype(np.float64) @ Bm.astype(np.float64)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    dD = torch.full((128, N), float("nan"), device="cuda")
    lib = _lib.load()
    _lib.check("gdn_selftest_umma", lib.gdn_selftest_umma(mode, dA.data_ptr(), dB.data_ptr(), dD.data_ptr(), None))
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    D = dD.cpu().numpy()
    # tf32 operands: ~2^-11 relative rounding per element, sum of K products;
    # bf16 operands are exact after the rounding above: fp32 accumulation only
    tol = 1e-3 if mode in BF16_MODES else 4.0 * 2.0 ** -11 * np.sqrt(K) * 3.0
    err = np.abs(D - ref).max()
    assert np.isfinite(D).all() and err < tol, f"mode {mode}: max err {err}"
