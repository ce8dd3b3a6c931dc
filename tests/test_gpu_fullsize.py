"""Parity at the benchmark workloads' full sizes.

* Chunked prefill, batch 8 x 8192 tokens, 16 key / 32 value heads, d 128,
  bf16 (the prefill benchmark's inputs: x ~ N(0, 1) from the device generator
  seeded 3, projected by the layer): rows 0 and 7 are compared with the oracle
  (all 32 heads, all 8192 tokens, i.e. 128 chunks per chain) at the flat
  tolerances: outputs within 2e-2 (or one bf16 ulp where that is larger),
  final state within 1e-3 max relative error, conv state bit-exact.  The rows
  of a batch are independent, so two rows pin the whole call.
* The same call through properties that hold at any size: splitting the
  sequence at T/2 and handing the states over gives the same result as one
  call, and the conv state at the split equals the conv checkpoint bit for bit.
* Decode, batch 64: 512 single-token steps from pre-filled states
  (S0 ~ N(0, 0.02^2)), every step's projection outputs from x ~ N(0, 1);
  rows 0, 31 and 63 follow the oracle step by step (outputs of every step,
  final recurrent and conv states).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gdn_oracle as O
from tests.helpers import assert_bf16_close, assert_bit_exact, assert_state_close
from tests.test_gpu_mixer import make_layer
from visionstack_b200 import workloads as W

pytestmark = pytest.mark.gpu

B, T = 8, 8192


@pytest.fixture(scope="module")
def full_inputs():
    shape = W.SHAPE_QWEN
    m, params = make_layer(shape, "bf16")
    dev = torch.device("cuda")
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    with torch.no_grad():
        x = torch.randn(B, T, shape.hidden_size, generator=g, device=dev).to(torch.bfloat16)
        mixed, z, bb, aa = m.project(x)
        del x
    return m, params, shape, mixed, z, bb, aa


def _np(t: torch.Tensor) -> np.ndarray:
    return t.float().cpu().numpy()


def test_full_size_prefill_rows_match_oracle(full_inputs):
    from visionstack_b200 import _lib
    m, params, shape, mixed, z, bb, aa = full_inputs
    dev = mixed.device
    S = torch.empty(B, shape.num_v_heads, shape.head_k_dim, shape.head_v_dim, device=dev)
    cs = torch.empty(B, shape.conv_dim, shape.conv_kernel - 1, dtype=torch.bfloat16, device=dev)
    out = m.mixer(mixed, z, bb, aa, conv_state_out=cs, rec_state_out=S, token_by_token=False)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    for row in (0, B - 1):
        r_out, r_cs, r_S, _, _ = O.mixer_forward(
            shape, _np(mixed[row:row + 1]), _np(z[row:row + 1]).reshape(1, T, shape.num_v_heads, shape.head_v_dim),
            _np(aa[row:row + 1]), _np(bb[row:row + 1]), params["conv1d.weight"], params["A_log"],
            params["dt_bias"], params["norm.weight"], "bf16", chunk=True)
        what = f"prefill B8 x T8192 row {row}"
        assert_bit_exact(cs[row:row + 1], r_cs, what + " conv state")
        assert_state_close(S[row:row + 1], r_S, what + " final state", report=True)
        assert_bf16_close(out[row:row + 1], r_out, what + " outputs", report=True)


def test_full_size_prefill_composes_over_a_split(full_inputs):
    from visionstack_b200 import _lib
    m, _, shape, mixed, z, bb, aa = full_inputs
    dev = mixed.device
    h = T // 2
    S_full = torch.empty(B, shape.num_v_heads, shape.head_k_dim, shape.head_v_dim, device=dev)
    cs_full = torch.empty(B, shape.conv_dim, shape.conv_kernel - 1, dtype=torch.bfloat16, device=dev)
    st_ck = torch.empty(1, *S_full.shape, device=dev)
    cv_ck = torch.empty(1, *cs_full.shape, dtype=torch.bfloat16, device=dev)
    out_full = m.mixer(mixed, z, bb, aa, conv_state_out=cs_full, rec_state_out=S_full, checkpoint_offsets=(h,),
                       state_checkpoints=st_ck, conv_checkpoints=cv_ck, token_by_token=False)
    S_half = torch.empty_like(S_full)
    cs_half = torch.empty_like(cs_full)
    out_a = m.mixer(mixed[:, :h], z[:, :h], bb[:, :h], aa[:, :h], conv_state_out=cs_half, rec_state_out=S_half,
                    token_by_token=False)
    S_end = torch.empty_like(S_full)
    cs_end = torch.empty_like(cs_full)
    out_b = m.mixer(mixed[:, h:], z[:, h:], bb[:, h:], aa[:, h:], conv_state=cs_half, rec_state=S_half,
                    conv_state_out=cs_end, rec_state_out=S_end, token_by_token=False)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert torch.isfinite(S_full).all() and torch.isfinite(out_full.float()).all()
    assert_bit_exact(cs_half, cv_ck[0], "conv state at the split = conv checkpoint")
    assert_bit_exact(cs_end, cs_full, "final conv state")
    assert_state_close(S_half, st_ck[0], "state at the split = state checkpoint", scale=2.0)
    assert_state_close(S_end, S_full, "final state over a split", scale=2.0)
    assert_bf16_close(out_a, out_full[:, :h], "outputs of the first half")
    assert_bf16_close(out_b, out_full[:, h:], "outputs of the second half", scale=2.0)


def test_full_size_prefill_forms_agree(full_inputs):
    """The default two-kernel form, the prep-in-kernel single kernel and the older single kernel on the
    same call."""
    from visionstack_b200 import _lib
    m, _, shape, mixed, z, bb, aa = full_inputs
    dev = mixed.device
    res = []
    for kw in ({}, {"prep_in_kernel_prefill": True}, {"fused_prefill": True}):
        S = torch.empty(B, shape.num_v_heads, shape.head_k_dim, shape.head_v_dim, device=dev)
        o = m.mixer(mixed, z, bb, aa, rec_state_out=S, token_by_token=False, **kw)
        res.append((o, S))
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    for i, name in ((1, "prep-in-kernel"), (2, "single-kernel")):
        assert_state_close(res[0][1], res[i][1], f"default vs {name} final state", scale=2.0)
        assert_bf16_close(res[0][0], res[i][0], f"default vs {name} outputs", scale=2.0)


def test_decode_512_steps_match_oracle():
    """The decode workload: B64, 512 single-token steps, states updated in place."""
    from visionstack_b200 import _lib
    wl = W.WORKLOADS["decode"]
    shape = wl.shape
    m, params = make_layer(shape, "bf16")
    dev = torch.device("cuda")
    st = W.make_decode_states(wl)
    S = torch.from_numpy(st["recurrent"]).to(dev)
    convs = [torch.from_numpy(st["conv"]).to(dev).to(torch.bfloat16),
             torch.empty(wl.batch, shape.conv_dim, shape.conv_kernel - 1, dtype=torch.bfloat16, device=dev)]
    rows = [0, 31, 63]
    g = torch.Generator(device=dev)
    g.manual_seed(wl.x_seed)
    ins, outs = [], []
    with torch.no_grad():
        for i in range(wl.steps):
            x = torch.randn(wl.batch, 1, shape.hidden_size, generator=g, device=dev).to(torch.bfloat16)
            mixed, z, bb, aa = m.project(x)
            out = m.mixer(mixed, z, bb, aa, conv_state=convs[i % 2], rec_state=S, conv_state_out=convs[(i + 1) % 2],
                          rec_state_out=S, token_by_token=True)
            ins.append(tuple(_np(t[rows]) for t in (mixed, z, aa, bb)))
            outs.append(_np(out[rows]))
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    r_conv = st["conv"][rows]
    r_S = st["recurrent"][rows]
    worst = 0.0
    for i in range(wl.steps):
        mx, zz, a_, b_ = ins[i]
        r_out, r_conv, r_S, _, _ = O.mixer_forward(
            shape, mx, zz.reshape(len(rows), 1, shape.num_v_heads, shape.head_v_dim), a_, b_,
            params["conv1d.weight"], params["A_log"], params["dt_bias"], params["norm.weight"], "bf16",
            r_conv, r_S, chunk=False)
        assert_bf16_close(outs[i], r_out, f"decode step {i} outputs")
        worst = max(worst, float(np.max(np.abs(outs[i].astype(np.float64) - r_out.astype(np.float64)))))
    assert_bit_exact(convs[wl.steps % 2][rows], r_conv, "conv state after 512 steps")
    assert_state_close(S[rows], r_S, "decode B64 x 512 steps, rows 0/31/63: final state", report=True)
    from tests.helpers import PARITY_REPORT
    PARITY_REPORT.append(f"decode B64 x 512 steps, rows 0/31/63: max |err| of the outputs over all steps {worst:.4g}")
