"""The fused elementwise steps of the stack's layers (csrc/stack_ops.cu) against PyTorch's own ops
on the same bf16 inputs: the zero-centred RMSNorm (config.py:118-127) on contiguous and strided
rows (the per-head q norm reads every other 256-element run of the query projection), with and
without the residual add in front (text.py:233-276; the residual itself bit-exact), and the MLP's
SiLU(gate) * up with torch's two roundings (text.py:215-230)."""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _ref_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * (1.0 + w.float())).to(x.dtype)


def _within_one_rounding(y: torch.Tensor, ref_f32: torch.Tensor, what: str):
    rb = ref_f32.to(torch.bfloat16).float()
    tol = torch.maximum(rb.abs() * 2.0 ** -7, torch.full_like(rb, 1e-30))
    bad = int(((y.float() - ref_f32).abs() > tol).sum())
    assert bad == 0, f"{what}: {bad} elements off by more than one bf16 rounding"


@pytest.mark.parametrize("shape", [(32, 1, 2048), (3, 4099, 2048), (5, 7, 256)])
def test_rms_norm_matches_reference(shape):
    from visionstack_b200.stack import Qwen3_5RMSNorm
    g = torch.Generator(device="cuda")
    g.manual_seed(sum(shape))
    n = Qwen3_5RMSNorm(shape[-1]).cuda().to(torch.bfloat16)
    with torch.no_grad():
        n.weight.copy_(0.1 * torch.randn(shape[-1], generator=g, device="cuda"))
        x = (3.0 * torch.randn(*shape, generator=g, device="cuda")).to(torch.bfloat16)
        y = n(x)
        xf = x.float()
        ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + n.eps) * (1.0 + n.weight.float())
    assert n._kernel_ok(x)
    _within_one_rounding(y, ref, f"norm {shape}")


def test_rms_norm_on_strided_head_rows():
    """q = the first 256 of every 512 values per head (query and gate interleaved per head)."""
    from visionstack_b200.stack import Qwen3_5RMSNorm
    g = torch.Generator(device="cuda")
    g.manual_seed(1)
    B, T, H, hd = 2, 3, 16, 256
    qg = torch.randn(B, T, H, 2 * hd, generator=g, device="cuda").to(torch.bfloat16)
    q = qg[..., :hd]
    n = Qwen3_5RMSNorm(hd).cuda().to(torch.bfloat16)
    with torch.no_grad():
        n.weight.copy_(0.1 * torch.randn(hd, generator=g, device="cuda"))
        y = n(q)
        qf = q.float()
        ref = qf * torch.rsqrt(qf.pow(2).mean(-1, keepdim=True) + n.eps) * (1.0 + n.weight.float())
    assert n._kernel_ok(q) and y.shape == q.shape and y.is_contiguous()
    _within_one_rounding(y, ref, "strided head rows")


def test_residual_add_and_norm():
    from visionstack_b200.stack import Qwen3_5RMSNorm
    g = torch.Generator(device="cuda")
    g.manual_seed(2)
    n = Qwen3_5RMSNorm(2048).cuda().to(torch.bfloat16)
    with torch.no_grad():
        n.weight.copy_(0.1 * torch.randn(2048, generator=g, device="cuda"))
        x = torch.randn(32, 1, 2048, generator=g, device="cuda").to(torch.bfloat16)
        d = torch.randn(32, 1, 2048, generator=g, device="cuda").to(torch.bfloat16)
        h, y = n.add_forward(x, d)
        href = x + d
        hf = href.float()
        ref = hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + n.eps) * (1.0 + n.weight.float())
    assert torch.equal(h, href), "the residual stream must be x + delta in bf16, bit for bit"
    _within_one_rounding(y, ref, "residual + norm")


def test_silu_mul_matches_torch():
    from visionstack_b200.stack import Qwen3_5MLP
    from visionstack_b200 import Qwen3_5TextConfig
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    cfg = Qwen3_5TextConfig(hidden_size=256)
    mlp = Qwen3_5MLP(cfg, 512).cuda().to(torch.bfloat16)
    x = torch.randn(4, 1, 256, generator=g, device="cuda").to(torch.bfloat16)
    with torch.no_grad():
        y = mlp(x)
        gt, up = F.linear(x, mlp.gate_proj.weight), F.linear(x, mlp.up_proj.weight)
        ref = F.linear(F.silu(gt) * up, mlp.down_proj.weight)
    # identical activations into down_proj up to the last bit of silu: compare the outputs closely
    assert float((y.float() - ref.float()).abs().max()) <= 2.0 ** -6 * float(ref.float().abs().max())
    from visionstack_b200 import _lib
    a = (4.0 * torch.randn(1 << 16, generator=g, device="cuda")).to(torch.bfloat16)
    b = torch.randn(1 << 16, generator=g, device="cuda").to(torch.bfloat16)
    out = torch.empty_like(a)
    _lib.check("silu_mul", _lib.load().gdn_silu_mul(a.data_ptr(), b.data_ptr(), out.data_ptr(), a.numel(), None))
    torch.cuda.synchronize()
    r = F.silu(a) * b
    diff = (out.float() - r.float()).abs()
    assert int((diff > 0).sum()) <= a.numel() // 1000, "more than 0.1% of the elements differ from torch's"
    assert bool((diff <= r.float().abs() * 2.0 ** -7 + 1e-30).all())


def test_qk_norm_rope_and_gate_match_torch():
    """The attention's fused steps against torch's ops on the same bf16 tensors: q / k norms and
    the partial rotary embedding (head dim 256, 64 rotary channels as in the stack), and the gated
    output for a contiguous and a transposed (flash-attention-like) attention output."""
    from visionstack_b200 import Qwen3_5TextConfig
    from visionstack_b200.stack import Qwen3_5Attention, Qwen3_5TextRotaryEmbedding, _apply_rotary_pos_emb_partial
    g = torch.Generator(device="cuda")
    g.manual_seed(4)
    cfg = Qwen3_5TextConfig(hidden_size=512, num_attention_heads=4, num_key_value_heads=2, head_dim=256)
    attn = Qwen3_5Attention(cfg, 3).cuda().to(torch.bfloat16)
    B, T, hd = 2, 5, 256
    with torch.no_grad():
        attn.q_norm.weight.copy_(0.1 * torch.randn(hd, generator=g, device="cuda"))
        attn.k_norm.weight.copy_(0.1 * torch.randn(hd, generator=g, device="cuda"))
        qg = torch.randn(B, T, 4, 2 * hd, generator=g, device="cuda").to(torch.bfloat16)
        kr = torch.randn(B, T, 2, hd, generator=g, device="cuda").to(torch.bfloat16)
        pos = (torch.arange(T, device="cuda") + 37)[None, None].expand(3, B, T)
        cos, sin = Qwen3_5TextRotaryEmbedding(cfg)(qg, pos)
        assert attn._fused_ok(qg, kr, cos, sin)
        q, k = attn._qk_norm_rope(qg, kr, cos, sin)
        qn = _ref_norm(qg[..., :hd], attn.q_norm.weight, attn.q_norm.eps).transpose(1, 2)
        kn = _ref_norm(kr, attn.k_norm.weight, attn.k_norm.eps).transpose(1, 2)
        rq, rk = _apply_rotary_pos_emb_partial(qn, kn, cos, sin)
    assert q.shape == rq.shape and k.shape == rk.shape
    for got, ref, name in ((q, rq, "q"), (k, rk, "k")):
        d = (got.float() - ref.float()).abs()
        # the norm's mean is summed in another order: a normed value may round to the
        # neighbouring bf16, which the rotation carries (at most a couple of roundings)
        assert bool((d <= ref.float().abs() * 2.0 ** -6 + 2.0 ** -12).all()), f"{name}: max diff {float(d.max())}"
        assert int((d > 0).sum()) <= ref.numel() // 100, f"{name}: too many elements differ"
    with torch.no_grad():
        for o in (torch.randn(B, 4, T, hd, generator=g, device="cuda").to(torch.bfloat16),
                  torch.randn(B, T, 4, hd, generator=g, device="cuda").to(torch.bfloat16).transpose(1, 2)):
            out = attn._gated(o, qg, None)
            ref = o.transpose(1, 2).reshape(B, T, -1).contiguous() * torch.sigmoid(qg[..., hd:].reshape(B, T, -1))
            d = (out.float() - ref.float()).abs()
            assert bool((d <= ref.float().abs() * 2.0 ** -7 + 1e-30).all())
            assert int((d > 0).sum()) <= ref.numel() // 1000
