"""Tolerances and comparison helpers shared by the parity tests.

Tolerances (the path's parity bar):
* outputs in bf16: |ours - ref| <= 2e-2, or at most one bf16 ulp of the
  reference value (2^-7 |ref|) where that ulp is larger than 2e-2 (|ref| > 2.56):
  two correct fp32 pipelines may round a large output to neighbouring bf16
  values;
* outputs in fp32: |ours - ref| <= 1e-4 (layer level) / 5e-5 (mixer level);
* recurrent states (fp32): max |ours - ref| / max |ref| <= 1e-3;
* conv states, conv checkpoints, checkpoint keys: bit-exact.
"""
from __future__ import annotations

import numpy as np

BF16_ABS = 2e-2
STATE_REL = 1e-3

# Comparisons made with ``report=True``: printed in the terminal summary of the
# run (strict max-abs error, elements that needed the one-ulp rule, state error).
PARITY_REPORT = []


def to_np(t) -> np.ndarray:
    if hasattr(t, "detach"):
        return t.detach().float().cpu().numpy()
    return np.asarray(t, dtype=np.float32)


def max_abs(a, b) -> float:
    return float(np.max(np.abs(to_np(a).astype(np.float64) - to_np(b).astype(np.float64))))


def rel_max(a, b) -> float:
    b = to_np(b)
    return max_abs(a, b) / max(1e-30, float(np.max(np.abs(b))))


def assert_bf16_close(ours, ref, what="", scale=1.0, report=False):
    """``scale`` = 2 compares two implementations that are each within the
    tolerance of the reference."""
    o, r = to_np(ours).astype(np.float64), to_np(ref).astype(np.float64)
    assert o.shape == r.shape, (what, o.shape, r.shape)
    err = np.abs(o - r)
    lim = scale * np.maximum(BF16_ABS, np.abs(r) * 2.0 ** -7)
    bad = err > lim
    if report:
        n_ulp = int(np.count_nonzero(err > scale * BF16_ABS))
        PARITY_REPORT.append(f"{what}: max |err| {float(err.max()):.4g} over {err.size} elements (flat bar "
                             f"{scale * BF16_ABS:g}); {n_ulp} elements above the flat bar, within one bf16 ulp "
                             f"of the reference; {int(bad.sum())} outside tolerance")
    assert not bad.any(), (f"{what}: {int(bad.sum())} elements outside tolerance, worst err "
                           f"{float(err.max()):.3g} (ref {float(r.flat[int(np.argmax(err))]):.3g})")


def assert_f32_close(ours, ref, tol, what=""):
    err = max_abs(ours, ref)
    assert err <= tol, f"{what}: max abs err {err:.3g} > {tol}"


def assert_state_close(ours, ref, what="", tol=STATE_REL, scale=1.0, report=False):
    tol = tol * scale
    err = rel_max(ours, ref)
    if report:
        PARITY_REPORT.append(f"{what}: state max|err|/max|ref| {err:.3g} (bar {tol:g})")
    assert err <= tol, f"{what}: state max rel err {err:.3g} > {tol}"


def assert_bit_exact(ours, ref, what=""):
    o, r = to_np(ours), to_np(ref)
    assert o.shape == r.shape, (what, o.shape, r.shape)
    assert np.array_equal(o, r), f"{what}: {int((o != r).sum())} elements differ"
