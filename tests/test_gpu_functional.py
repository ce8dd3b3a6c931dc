"""Functional names of the reference module backed by stand-alone kernels:
``_solve_unit_lower_triangular`` / ``_invert_unit_lower_triangular_block``
(deltanet.py:93-162) and ``Qwen3_5RMSNormGated.forward`` (config.py:136-143).

The triangular-solve checks restate the reference's own self-test
(ShadowBoxer/sanitycheck/gate3_models.py:1169-1191: a split right-hand side
gives the same solution as the concatenated one, and the residual of the
system is small) and compare with fixtures recorded from the reference
(``tests/golden/solve.npz``)."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import gdn_oracle as O
from tests.helpers import assert_bf16_close, assert_f32_close
from visionstack_b200 import Qwen3_5RMSNormGated, _invert_unit_lower_triangular_block, _solve_unit_lower_triangular

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_solver_self_test_of_the_reference():
    """gate3_models.py:1169-1191 on the CUDA solver: cat_diff < 1e-5, residual < 1e-4."""
    dev = torch.device("cuda")
    g = torch.Generator(device=dev)
    g.manual_seed(1234)
    ut = torch.randn((1, 2, 1, 64, 64), generator=g, device=dev).tril(-1) * 0.05
    ut = ut + torch.eye(64, device=dev)
    rhs_a = torch.randn((1, 2, 1, 64, 32), generator=g, device=dev)
    rhs_b = torch.randn((1, 2, 1, 64, 32), generator=g, device=dev)
    sol_a = _solve_unit_lower_triangular(ut, rhs_a)
    sol_b = _solve_unit_lower_triangular(ut, rhs_b)
    cat_a, cat_b = torch.split(_solve_unit_lower_triangular(ut, torch.cat([rhs_a, rhs_b], dim=-1)), [32, 32], dim=-1)
    tri_diff = max(float((sol_a - cat_a).abs().max()), float((sol_b - cat_b).abs().max()))
    res_err = float(((ut @ sol_a) - rhs_a).abs().max())
    assert tri_diff < 1e-5 and res_err < 1e-4, (tri_diff, res_err)


@pytest.mark.parametrize("n", [16, 20, 32, 64])
def test_solver_matches_reference_fixtures(n):
    d = np.load(GOLDEN / "solve.npz")
    ut = torch.from_numpy(d[f"ut{n}"]).cuda()
    rhs = torch.from_numpy(d[f"rhs{n}"]).cuda()
    sol = _solve_unit_lower_triangular(ut, rhs)
    assert sol.shape == rhs.shape and sol.dtype == torch.float32
    assert_f32_close(sol, d[f"sol{n}"], 2e-5, f"solve n={n}")


@pytest.mark.parametrize("n", [16, 32, 64, 128, 130])
def test_block_inverse_matches_oracle(n):
    rng = np.random.default_rng(n)
    u = (0.1 * rng.standard_normal((3, 2, n, n))).astype(np.float32)
    ours = _invert_unit_lower_triangular_block(torch.from_numpy(u).cuda())
    ref = O.invert_unit_lower_triangular_block(u)
    assert_f32_close(ours, ref, 5e-5, f"inverse n={n}")
    # (I + tril(u, -1)) @ inverse == I
    eye = np.eye(n, dtype=np.float32)
    prod = (eye + np.tril(u, -1)) @ ours.cpu().numpy()
    assert_f32_close(prod, np.broadcast_to(eye, prod.shape), 1e-4, f"inverse residual n={n}")


def test_solver_broadcasts_batch_dims_and_keeps_dtype():
    rng = np.random.default_rng(7)
    u = (0.1 * rng.standard_normal((1, 4, 32, 32))).astype(np.float32)
    r = rng.standard_normal((3, 4, 32, 5)).astype(np.float32)
    ours = _solve_unit_lower_triangular(torch.from_numpy(u).cuda(), torch.from_numpy(r).cuda())
    ref = O.solve_unit_lower_triangular(np.broadcast_to(u, (3, 4, 32, 32)).copy(), r)
    assert ours.shape == (3, 4, 32, 5)
    assert_f32_close(ours, ref, 5e-5, "broadcast solve")


@pytest.mark.parametrize("x_dt,w_dt,g_dt", [("bf16", "bf16", "bf16"), ("f32", "f32", "f32"),
                                             ("bf16", "f32", "bf16"), ("bf16", "bf16", "f32")])
def test_rms_norm_gated_forward_matches_oracle(x_dt, w_dt, g_dt):
    tdt = {"bf16": torch.bfloat16, "f32": torch.float32}
    rng = np.random.default_rng(11)
    rows, dim = 777, 128
    x = (1.5 * rng.standard_normal((3, rows // 3 + 1, dim))).astype(np.float32)
    z = (1.5 * rng.standard_normal(x.shape)).astype(np.float32)
    w = (1.0 + 0.3 * rng.standard_normal(dim)).astype(np.float32)
    xt = torch.from_numpy(x).cuda().to(tdt[x_dt])
    zt = torch.from_numpy(z).cuda().to(tdt[g_dt])
    norm = Qwen3_5RMSNormGated(dim, eps=1e-6).cuda()
    with torch.no_grad():
        norm.weight.data = torch.from_numpy(w).cuda().to(tdt[w_dt])
    out = norm(xt, zt)
    assert out.dtype == xt.dtype and out.shape == xt.shape
    # the oracle's inputs are the values the kernel sees (rounded to their dtypes)
    xr = xt.float().cpu().numpy()
    zr = zt.float().cpu().numpy()
    wr = norm.weight.detach().float().cpu().numpy()
    prod_dtype = "bf16" if (x_dt == "bf16" and w_dt == "bf16") else "f32"
    ref = O.rms_norm_gated(xr.reshape(-1, dim), zr.reshape(-1, dim), wr, 1e-6, x_dt) if prod_dtype == x_dt else None
    if ref is None:  # bf16 input with an fp32 weight: the weight product stays fp32
        hf = xr.reshape(-1, dim)
        var = np.mean(hf * hf, axis=-1, keepdims=True, dtype=np.float32)
        normed = O.cast(hf * (np.float32(1.0) / np.sqrt(var + np.float32(1e-6))), x_dt)
        ref = O.cast((wr * normed) * O.silu(zr.reshape(-1, dim)), x_dt)
    if x_dt == "bf16":
        assert_bf16_close(out.reshape(-1, dim), ref, "gated norm")
    else:
        assert_f32_close(out.reshape(-1, dim), ref, 1e-5, "gated norm")


def test_rms_norm_gated_rejects_cpu_tensors():
    norm = Qwen3_5RMSNormGated(8)
    with pytest.raises(RuntimeError, match="CUDA"):
        norm(torch.zeros(2, 8), torch.zeros(2, 8))
