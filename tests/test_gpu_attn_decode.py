"""The decode-attention kernel of the hybrid stack's full-attention layers (gdn_attn_decode)
against fp32 SDPA on the valid keys: one query token per row, grouped-query, keys 0..pos of a
fixed-capacity buffer, pos read on the device.  bf16 output: max abs error 1e-2 (outputs are
weighted means of N(0,1) values; one bf16 ulp at 1 is 0.008)."""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from visionstack_b200.stack import _decode_attention

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("hd", [64, 128, 256])
@pytest.mark.parametrize("groups", [1, 2, 4, 8])
def test_decode_attention_matches_sdpa(hd, groups):
    dev = torch.device("cuda")
    g = torch.Generator(device=dev)
    g.manual_seed(hd * 10 + groups)
    B, KVH, cap = 3, 2, 300
    q = torch.randn(B, KVH * groups, 1, hd, generator=g, device=dev).to(torch.bfloat16)
    kb = torch.randn(B, KVH, cap, hd, generator=g, device=dev).to(torch.bfloat16)
    vb = torch.randn(B, KVH, cap, hd, generator=g, device=dev).to(torch.bfloat16)
    scale = hd ** -0.5
    for last in (0, 31, 32, 200, 299, 5000):
        pos = torch.tensor([last], dtype=torch.long, device=dev)
        o = _decode_attention(q, kb, vb, pos, scale)
        n = min(cap, last + 1)
        ref = F.scaled_dot_product_attention(q.float(), kb[:, :, :n].float(), vb[:, :, :n].float(), scale=scale,
                                             enable_gqa=True)
        torch.cuda.synchronize()
        err = (o.float() - ref).abs().max().item()
        assert err <= 1e-2, f"hd {hd} groups {groups} pos {last}: {err:.3e}"


def test_decode_attention_full_size_shape():
    dev = torch.device("cuda")
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    B, KVH, G, hd, cap, last = 32, 2, 8, 256, 4352, 4100
    q = torch.randn(B, KVH * G, 1, hd, generator=g, device=dev).to(torch.bfloat16)
    kb = torch.randn(B, KVH, cap, hd, generator=g, device=dev).to(torch.bfloat16)
    vb = torch.randn(B, KVH, cap, hd, generator=g, device=dev).to(torch.bfloat16)
    pos = torch.tensor([last], dtype=torch.long, device=dev)
    o = _decode_attention(q, kb, vb, pos, hd ** -0.5)
    ref = F.scaled_dot_product_attention(q.float(), kb[:, :, :last + 1].float(), vb[:, :, :last + 1].float(),
                                         scale=hd ** -0.5, enable_gqa=True)
    assert (o.float() - ref).abs().max().item() <= 1e-2
