"""The chunked prefill at the prefill benchmark's full size (batch 8 x 8192 tokens,
16 key / 32 value heads, d 128, bf16), where the oracle would take hours: checked
through properties that hold at any size.

* Splitting the sequence: prefill of tokens [0, T/2) with its final conv and
  recurrent state handed to a prefill of [T/2, T) gives the same outputs and final
  state as one prefill of [0, T) (the chunk recurrence composes), and the handed
  conv state equals the conv checkpoint at T/2 bit for bit.
* An independent implementation: the single fused tensor-core kernel agrees with
  the two-kernel path (each within tolerance of the reference, so with twice the
  tolerance of each other).
"""
from __future__ import annotations

import pytest
import torch

from tests.helpers import assert_bf16_close, assert_bit_exact, assert_state_close
from tests.test_gpu_mixer import make_layer
from visionstack_b200 import workloads as W

pytestmark = pytest.mark.gpu

B, T = 8, 8192


@pytest.fixture(scope="module")
def full_inputs():
    shape = W.SHAPE_QWEN
    m, _ = make_layer(shape, "bf16")
    dev = torch.device("cuda")
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    with torch.no_grad():
        x = torch.randn(B, T, shape.hidden_size, generator=g, device=dev).to(torch.bfloat16)
        mixed, z, bb, aa = m.project(x)
    return m, shape, mixed, z, bb, aa


def test_full_size_prefill_composes_over_a_split(full_inputs):
    from visionstack_b200 import _lib
    m, shape, mixed, z, bb, aa = full_inputs
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


def test_full_size_two_kernel_matches_fused_kernel(full_inputs):
    from visionstack_b200 import _lib
    m, shape, mixed, z, bb, aa = full_inputs
    dev = mixed.device
    res = []
    for kw in ({}, {"fused_prefill": True}):
        S = torch.empty(B, shape.num_v_heads, shape.head_k_dim, shape.head_v_dim, device=dev)
        o = m.mixer(mixed, z, bb, aa, rec_state_out=S, token_by_token=False, **kw)
        res.append((o, S))
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert_state_close(res[0][1], res[1][1], "two-kernel vs fused final state", scale=2.0)
    assert_bf16_close(res[0][0], res[1][0], "two-kernel vs fused outputs", scale=2.0)
