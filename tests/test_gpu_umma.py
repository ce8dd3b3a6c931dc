"""The tensor-core building blocks of the chunked kernel (tcgen05 MMA with
tf32 operands from 128-byte swizzled shared memory, fp32 accumulation in
tensor memory) against a float64 host matmul, for every operand layout the
chunked kernel uses."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from visionstack_b200 import _lib

pytestmark = pytest.mark.gpu

# mode: (K, N, A MN-major, B MN-major); modes 4-6 read A from tensor memory
SHAPES = {0: (128, 64, False, False), 1: (128, 128, False, True), 2: (64, 128, False, True),
          3: (64, 128, True, True), 4: (128, 128, False, False), 5: (64, 64, False, False),
          6: (64, 128, False, True)}


@pytest.mark.parametrize("mode", sorted(SHAPES))
def test_umma_layouts(mode):
    K, N, a_mn, b_mn = SHAPES[mode]
    rng = np.random.default_rng(mode)
    A = rng.standard_normal((K, 128) if a_mn else (128, K)).astype(np.float32)
    B = rng.standard_normal((N, K) if not b_mn else (K, N)).astype(np.float32)
    Am = A.T if a_mn else A
    Bm = B.T if not b_mn else B
    ref = Am.astype(np.float64) @ Bm.astype(np.float64)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    dD = torch.full((128, N), float("nan"), device="cuda")
    lib = _lib.load()
    _lib.check("gdn_selftest_umma", lib.gdn_selftest_umma(mode, dA.data_ptr(), dB.data_ptr(), dD.data_ptr(), None))
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    D = dD.cpu().numpy()
    # tf32 operands: ~2^-11 relative rounding per element, sum of K products
    tol = 4.0 * 2.0 ** -11 * np.sqrt(K) * 3.0
    err = np.abs(D - ref).max()
    assert np.isfinite(D).all() and err < tol, f"mode {mode}: max err {err}"
