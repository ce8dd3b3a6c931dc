"""The hybrid decoder stack around the token mixer: a harness for the 48-layer workload.

Mirrors ShadowBoxer/models/qwen35/text.py (class names, parameter names, forward contracts and
cache side effects) so a reference state dict loads unchanged: every `linear_attention` layer is
this package's `Qwen3_5GatedDeltaNet` (the CUDA token mixer); the full-attention layers, the MLPs
and the norms are plain PyTorch with library kernels (cuBLAS GEMMs, SDPA attention).

One change of mechanism, not of result: the reference appends every step's keys and values to the
cache with `torch.cat` (text.py:170-178), copying the whole history per step.  Given a
`kv_capacity` on the cache, `Qwen3_5Attention` writes them into a per-layer buffer of that
capacity instead and stores views of the filled part under the same dict keys, so the cached
tensors hold the same values.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Optional, Tuple

import torch
import torch.nn.functional as F
from torch import nn

from .cache import Qwen3_5HybridCache
from .config import Qwen3_5TextConfig, _linear
from .deltanet import Qwen3_5GatedDeltaNet


def _rows(x: torch.Tensor) -> Optional[Tuple[int, int]]:
    """(rows, row stride) of ``x`` seen as rows of its last dimension, or None when its rows are not
    evenly spaced (the last dimension must be contiguous)."""
    if x.dim() < 2 or x.stride(-1) != 1:
        return None
    for i in range(x.dim() - 2):
        if x.stride(i) != x.stride(i + 1) * x.shape[i + 1]:
            return None
    return x.numel() // x.shape[-1], x.stride(-2)


def _bf16_kernel_ok(*ts: torch.Tensor) -> bool:
    return all(t.is_cuda and t.dtype == torch.bfloat16 and t.data_ptr() % 16 == 0 for t in ts)


def _rms_norm_zc(x: torch.Tensor, delta: Optional[torch.Tensor], w: torch.Tensor, eps: float):
    """The fused RMSNorm kernel (gdn_rms_norm_zc): returns (bf16(x + delta) or None, the norm)."""
    from . import _lib
    rx = _rows(x)
    rows, dim = rx[0], x.shape[-1]
    out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    res = torch.empty(x.shape, dtype=x.dtype, device=x.device) if delta is not None else None
    ds = _rows(delta)[1] if delta is not None else 0
    _lib.check("gdn_rms_norm_zc", _lib.load().gdn_rms_norm_zc(
        x.data_ptr(), rx[1], delta.data_ptr() if delta is not None else None, ds,
        res.data_ptr() if res is not None else None, w.data_ptr(), out.data_ptr(), rows, dim, float(eps),
        torch.cuda.current_stream(x.device).cuda_stream))
    return res, out


class Qwen3_5RMSNorm(nn.Module):
    """RMSNorm with a zero-centred weight, x / rms(x) * (1 + w), in fp32 (config.py:118-127).

    For bf16 CUDA tensors it runs the fused kernel ``gdn_rms_norm_zc`` (one launch instead of
    PyTorch's dtype copies, weight offset, norm and copy back); ``add_forward`` also fuses the
    decoder layer's residual add in front of it."""

    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.zeros(dim))

    def _kernel_ok(self, *ts: torch.Tensor) -> bool:
        dim = self.weight.shape[0]
        return (dim % 8 == 0 and self.weight.is_contiguous() and _bf16_kernel_ok(self.weight, *ts) and
                all(t.shape[-1] == dim and _rows(t) is not None and _rows(t)[1] % 8 == 0 for t in ts))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self._kernel_ok(x):
            return _rms_norm_zc(x, None, self.weight, self.eps)[1]
        # one fused normalisation kernel in fp32 (same math, one pass) instead of six elementwise ones
        w = 1.0 + self.weight.float()
        return F.rms_norm(x.float(), (x.shape[-1],), weight=w, eps=self.eps).to(x.dtype)

    def add_forward(self, x: torch.Tensor, delta: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """(x + delta, this norm of it), the residual stream kept in the activation dtype."""
        if x.shape == delta.shape and self._kernel_ok(x, delta):
            return _rms_norm_zc(x, delta, self.weight, self.eps)
        h = x + delta
        return h, self(h)


def _act(x: torch.Tensor, name: str) -> torch.Tensor:
    """The MLP activation by config name (config.py:99-106; unknown names fall back to SiLU)."""
    if name == "gelu_pytorch_tanh":
        return F.gelu(x, approximate="tanh")
    if name == "gelu":
        return F.gelu(x)
    return F.silu(x)


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


class Qwen3_5TextRotaryEmbedding(nn.Module):
    """Partial multimodal rotary embedding (text.py:25-73).

    `rotary = head_dim * partial_rotary_factor` channels rotate with inverse frequencies
    base^(-2i/rotary).  Positions come as [3, B, T] (temporal, height, width); frequency i takes
    the height position when i = 1 (mod 3) and i < 3 * mrope_section[1], the width position when
    i = 2 (mod 3) and i < 3 * mrope_section[2], the temporal position otherwise.  For text all
    three are equal.  cos / sin are [B, T, rotary] in the activation dtype.
    """

    def __init__(self, config: Qwen3_5TextConfig):
        super().__init__()
        rp = config.rope_parameters or {}
        self.base = float(rp.get("rope_theta", 10000000.0))
        head_dim = getattr(config, "head_dim", config.hidden_size // config.num_attention_heads)
        self.dim = int(head_dim * float(rp.get("partial_rotary_factor", 0.25)))
        self.mrope_section = list(rp.get("mrope_section", [11, 11, 10]))
        self._inv: Dict[torch.device, torch.Tensor] = {}

    def inv_freq(self, device: torch.device) -> torch.Tensor:
        t = self._inv.get(device)
        if t is None:  # computed on the host, then moved (as text.py:41-48 does)
            ex = torch.arange(0, self.dim, 2, dtype=torch.float32) / self.dim
            t = (1.0 / (self.base ** ex)).to(device)
            self._inv[device] = t
        return t

    def _select(self, f: torch.Tensor) -> torch.Tensor:
        # f [3, B, T, dim/2] -> [B, T, dim/2] with the sections' interleaved picks
        out = f[0].clone()
        n = f.shape[-1]
        for axis in (1, 2):
            idx = torch.arange(axis, min(n, 3 * self.mrope_section[axis]), 3, device=f.device)
            out[..., idx] = f[axis][..., idx]
        return torch.cat((out, out), dim=-1)

    @torch.no_grad()
    def forward(self, x: torch.Tensor, position_ids: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        pos = position_ids.expand(3, -1, -1).float()
        f = pos[..., None] * self.inv_freq(x.device)
        return self._select(f.cos()).to(x.dtype), self._select(f.sin()).to(x.dtype)


def _apply_rotary_pos_emb_partial(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor,
                                  sin: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Rotate the first `rotary` channels of q and k ([B, H, T, hd]); the rest pass (text.py:76-86)."""
    c, s = cos.unsqueeze(1), sin.unsqueeze(1)
    r = c.shape[-1]

    def rot(x: torch.Tensor) -> torch.Tensor:
        xr = x[..., :r]
        return torch.cat([xr * c + _rotate_half(xr) * s, x[..., r:]], dim=-1)

    return rot(q), rot(k)


def _decode_attention(q: torch.Tensor, kb: torch.Tensor, vb: torch.Tensor, pos: torch.Tensor,
                      scale: float) -> torch.Tensor:
    """One query token per row against fixed-capacity KV buffers on the CUDA decode-attention
    kernel (gdn_attn_decode): q [B, H, 1, hd], kb / vb [B, KVH, cap, hd] (bf16, contiguous), keys
    0..pos[0] (int64 on the device).  Returns [B, H, 1, hd]."""
    from . import _lib
    B, H, _, hd = q.shape
    kvh, cap = kb.shape[1], kb.shape[2]
    lib = _lib.load()
    n = int(lib.gdn_attn_decode_workspace_bytes(B, kvh, H // kvh, hd, cap))
    if n < 0:
        _lib.check("gdn_attn_decode_workspace_bytes", n)
    ws = torch.empty(n, dtype=torch.uint8, device=q.device)
    q = q.contiguous()
    out = torch.empty_like(q)
    _lib.check("gdn_attn_decode", lib.gdn_attn_decode(
        q.data_ptr(), kb.data_ptr(), vb.data_ptr(), pos.data_ptr(), out.data_ptr(), B, kvh, H // kvh, hd, cap,
        float(scale), ws.data_ptr(), n, torch.cuda.current_stream(q.device).cuda_stream))
    return out


def _kernel_decode_ok(q: torch.Tensor, kb: torch.Tensor) -> bool:
    g = q.shape[1] // kb.shape[1]
    return (q.is_cuda and q.dtype == torch.bfloat16 and kb.dtype == torch.bfloat16 and kb.is_contiguous() and
            q.shape[-1] in (64, 128, 256) and g in (1, 2, 4, 8) and q.shape[1] == g * kb.shape[1])


class Qwen3_5Attention(nn.Module):
    """Gated grouped-query attention (text.py:89-212): q_proj yields a query and a gate per head;
    q / k RMS-normalised per head, partial rotary, SDPA, output times sigmoid(gate), o_proj."""

    def __init__(self, config: Qwen3_5TextConfig, layer_idx: int):
        super().__init__()
        self.layer_idx = layer_idx
        self.head_dim = getattr(config, "head_dim", config.hidden_size // config.num_attention_heads)
        self.num_heads = config.num_attention_heads
        self.num_kv_heads = config.num_key_value_heads
        self.num_key_value_groups = self.num_heads // self.num_kv_heads
        self.scaling = self.head_dim ** -0.5
        hd, bias = self.head_dim, config.attention_bias
        self.q_proj = nn.Linear(config.hidden_size, self.num_heads * hd * 2, bias=bias)
        self.k_proj = nn.Linear(config.hidden_size, self.num_kv_heads * hd, bias=bias)
        self.v_proj = nn.Linear(config.hidden_size, self.num_kv_heads * hd, bias=bias)
        self.o_proj = nn.Linear(self.num_heads * hd, config.hidden_size, bias=bias)
        self.q_norm = Qwen3_5RMSNorm(hd, eps=config.rms_norm_eps)
        self.k_norm = Qwen3_5RMSNorm(hd, eps=config.rms_norm_eps)

    def _store_kv(self, cache: Qwen3_5HybridCache, k: torch.Tensor, v: torch.Tensor):
        """Append k, v ([B, kvh, T, hd]) to this layer's cache entry; returns the full history."""
        l = self.layer_idx
        pk, pv = cache.key_cache.get(l), cache.value_cache.get(l)
        has_past = pk is not None and pv is not None
        cap = int(getattr(cache, "kv_capacity", 0) or 0)
        if cap:
            bufs = cache.__dict__.setdefault("_kv_buffers", {})
            prev = pk.shape[2] if has_past else 0
            need = prev + k.shape[2]
            buf = bufs.get(l)
            ours = buf is not None and has_past and pk.data_ptr() == buf[0].data_ptr() and \
                pv.data_ptr() == buf[1].data_ptr()
            if buf is None or not (ours or not has_past) or buf[0].shape[2] < need or \
                    buf[0].shape[:2] != k.shape[:2] or buf[0].dtype != k.dtype:
                size = max(cap, need)
                # zeroed: the static decode path masks the unwritten tail, whose scores must be finite
                buf = (k.new_zeros(k.shape[0], k.shape[1], size, k.shape[3]),
                       v.new_zeros(v.shape[0], v.shape[1], size, v.shape[3]))
                if has_past:
                    buf[0][:, :, :prev].copy_(pk)
                    buf[1][:, :, :prev].copy_(pv)
                bufs[l] = buf
            buf[0][:, :, prev:need].copy_(k)
            buf[1][:, :, prev:need].copy_(v)
            k, v = buf[0][:, :, :need], buf[1][:, :, :need]
        elif has_past:
            k, v = torch.cat([pk, k], dim=2), torch.cat([pv, v], dim=2)
        cache.key_cache[l] = k
        cache.value_cache[l] = v
        return k, v, has_past

    def _static_decode(self, cache: Qwen3_5HybridCache, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                       pos: torch.Tensor, attention_mask: Optional[torch.Tensor]) -> torch.Tensor:
        """One decode token against this layer's fixed-capacity KV buffers with the position on
        the device (CUDA-graph capturable): k, v written at `pos`, attention over the keys 0..pos
        (the decode-attention kernel for bf16; otherwise SDPA over the whole buffer with the
        positions past `pos` masked out)."""
        if q.shape[2] != 1 or attention_mask is not None:
            raise ValueError("the static decode path takes one token and no attention mask")
        kb, vb = cache._kv_buffers[self.layer_idx]
        kb.index_copy_(2, pos, k)
        vb.index_copy_(2, pos, v)
        if _kernel_decode_ok(q, kb) and vb.is_contiguous():
            return _decode_attention(q, kb, vb, pos, self.scaling)
        cap = kb.shape[2]
        valid = (torch.arange(cap, device=q.device) <= pos).view(1, 1, 1, cap)
        B, hd = q.shape[0], self.head_dim
        G = self.num_key_value_groups
        o = F.scaled_dot_product_attention(q.reshape(B, self.num_kv_heads, G, hd), kb, vb, attn_mask=valid,
                                           scale=self.scaling)
        return o.reshape(B, self.num_heads, 1, hd)

    def _fused_ok(self, qg: torch.Tensor, kr: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> bool:
        hd, rot = self.head_dim, cos.shape[-1]
        ws = (self.q_norm.weight, self.k_norm.weight)
        return (hd % 8 == 0 and hd <= 256 and rot % 16 == 0 and rot <= hd and qg.is_contiguous() and
                kr.is_contiguous() and cos.is_contiguous() and sin.is_contiguous() and
                cos.shape == (qg.shape[0], qg.shape[1], rot) and sin.shape == cos.shape and
                all(w.is_contiguous() for w in ws) and _bf16_kernel_ok(qg, kr, cos, sin, *ws))

    def _qk_norm_rope(self, qg: torch.Tensor, kr: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
        """q / k norms and the partial rotary embedding in one launch (gdn_qk_norm_rope): q
        [B, H, T, hd] and k [B, KVH, T, hd], the layouts the torch path's rotation produces."""
        from . import _lib
        B, T, hd = qg.shape[0], qg.shape[1], self.head_dim
        q = torch.empty(B, self.num_heads, T, hd, dtype=qg.dtype, device=qg.device)
        k = torch.empty(B, self.num_kv_heads, T, hd, dtype=qg.dtype, device=qg.device)
        _lib.check("gdn_qk_norm_rope", _lib.load().gdn_qk_norm_rope(
            qg.data_ptr(), kr.data_ptr(), self.q_norm.weight.data_ptr(), self.k_norm.weight.data_ptr(),
            cos.data_ptr(), sin.data_ptr(), q.data_ptr(), k.data_ptr(), B, T, self.num_heads, self.num_kv_heads, hd,
            cos.shape[-1], float(self.q_norm.eps), torch.cuda.current_stream(qg.device).cuda_stream))
        return q, k

    def _gated(self, o: torch.Tensor, qg: torch.Tensor, gate: Optional[torch.Tensor]) -> torch.Tensor:
        """attn.transpose(1, 2).reshape(B, T, H hd) * sigmoid(gate) (text.py:204-209): one launch
        (gdn_attn_gate_out) when the fused path produced q, else torch's ops on ``gate``."""
        B, H, T, hd = o.shape
        if gate is None and o.stride(-1) == 1 and all(st % 8 == 0 for st in o.stride()[:3]) and \
                _bf16_kernel_ok(o, qg):
            from . import _lib
            out = torch.empty(B, T, H * hd, dtype=o.dtype, device=o.device)
            _lib.check("gdn_attn_gate_out", _lib.load().gdn_attn_gate_out(
                o.data_ptr(), o.stride(0), o.stride(1), o.stride(2), qg.data_ptr(), out.data_ptr(), B, T, H, hd,
                torch.cuda.current_stream(o.device).cuda_stream))
            return out
        if gate is None:
            gate = qg[..., hd:].reshape(B, T, H * hd)
        return o.transpose(1, 2).reshape(B, T, -1).contiguous() * torch.sigmoid(gate)

    def forward(self, hidden_states: torch.Tensor, position_embeddings: Tuple[torch.Tensor, torch.Tensor],
                attention_mask: Optional[torch.Tensor] = None,
                cache: Optional[Qwen3_5HybridCache] = None) -> torch.Tensor:
        B, T = hidden_states.shape[:2]
        hd = self.head_dim
        qg = _linear(self.q_proj, hidden_states).view(B, T, self.num_heads, 2 * hd)
        kr = _linear(self.k_proj, hidden_states).view(B, T, self.num_kv_heads, hd)
        v = _linear(self.v_proj, hidden_states).view(B, T, self.num_kv_heads, hd).transpose(1, 2)
        cos, sin = position_embeddings
        gate = None
        if self._fused_ok(qg, kr, cos, sin):
            q, k = self._qk_norm_rope(qg, kr, cos, sin)
        else:
            q, gate = qg[..., :hd], qg[..., hd:].reshape(B, T, self.num_heads * hd)
            q = self.q_norm(q).transpose(1, 2)
            k = self.k_norm(kr).transpose(1, 2)
            q, k = _apply_rotary_pos_emb_partial(q, k, cos, sin)
        static_pos = getattr(cache, "static_pos", None) if cache is not None else None
        if static_pos is not None:
            o = self._static_decode(cache, q, k, v, static_pos, attention_mask)
            return _linear(self.o_proj, self._gated(o, qg, gate))
        has_past = False
        if cache is not None:
            k, v, has_past = self._store_kv(cache, k, v)
        gqa = self.num_key_value_groups > 1
        kv_len = k.shape[2]
        bufs = getattr(cache, "_kv_buffers", {}) if cache is not None else {}
        buf = bufs.get(self.layer_idx)
        if attention_mask is None and has_past and T == 1 and buf is not None and \
                k.data_ptr() == buf[0].data_ptr() and v.data_ptr() == buf[1].data_ptr() and \
                _kernel_decode_ok(q, buf[0]) and buf[1].is_contiguous():
            pos = torch.tensor([kv_len - 1], dtype=torch.long, device=q.device)
            o = _decode_attention(q, buf[0], buf[1], pos, self.scaling)
        elif attention_mask is None and has_past and T == 1 and gqa:
            # one query per head: the query heads of one KV head become that head's queries
            # (the grouping of the GQA head expansion, h -> h // groups), so no K / V expansion
            G = self.num_key_value_groups
            o = F.scaled_dot_product_attention(q.reshape(B, self.num_kv_heads, G, hd), k, v, scale=self.scaling)
            o = o.reshape(B, self.num_heads, 1, hd)
        elif attention_mask is not None and attention_mask.ndim == 4:
            o = F.scaled_dot_product_attention(q, k, v, attn_mask=attention_mask, is_causal=False,
                                               scale=self.scaling, enable_gqa=gqa)
        elif has_past and T > 1:
            causal = torch.ones((T, kv_len), dtype=torch.bool, device=q.device).tril(diagonal=kv_len - T)
            o = F.scaled_dot_product_attention(q, k, v, attn_mask=causal[None, None], is_causal=False,
                                               scale=self.scaling, enable_gqa=gqa)
        else:
            o = F.scaled_dot_product_attention(q, k, v, is_causal=(T > 1 and not has_past), scale=self.scaling,
                                               enable_gqa=gqa)
        return _linear(self.o_proj, self._gated(o, qg, gate))


class Qwen3_5MLP(nn.Module):
    """Gated MLP down(act(gate(x)) * up(x)) (text.py:215-230)."""

    def __init__(self, config: Qwen3_5TextConfig, intermediate_size: int):
        super().__init__()
        self.gate_proj = nn.Linear(config.hidden_size, intermediate_size, bias=False)
        self.up_proj = nn.Linear(config.hidden_size, intermediate_size, bias=False)
        self.down_proj = nn.Linear(intermediate_size, config.hidden_size, bias=False)
        self.act_name = config.hidden_act

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        g, u = _linear(self.gate_proj, x), _linear(self.up_proj, x)
        if self.act_name not in ("gelu_pytorch_tanh", "gelu") and g.shape == u.shape and g.is_contiguous() and \
                u.is_contiguous() and g.numel() % 8 == 0 and _bf16_kernel_ok(g, u):
            from . import _lib
            h = torch.empty_like(g)  # act(gate) * up in one launch (gdn_silu_mul), torch's two roundings
            _lib.check("gdn_silu_mul", _lib.load().gdn_silu_mul(g.data_ptr(), u.data_ptr(), h.data_ptr(), g.numel(),
                                                               torch.cuda.current_stream(g.device).cuda_stream))
        else:
            h = _act(g, self.act_name) * u
        return _linear(self.down_proj, h)


class Qwen3_5DecoderLayer(nn.Module):
    """Pre-norm residual block: token mixer (DeltaNet or attention by `layer_types`), then the MLP
    (text.py:233-276)."""

    def __init__(self, config: Qwen3_5TextConfig, layer_idx: int):
        super().__init__()
        self.block_type = config.layer_types[layer_idx]
        if self.block_type == "linear_attention":
            self.linear_attn = Qwen3_5GatedDeltaNet(config, layer_idx)
        elif self.block_type == "full_attention":
            self.self_attn = Qwen3_5Attention(config, layer_idx)
        self.mlp = Qwen3_5MLP(config, config.intermediate_size)
        self.input_layernorm = Qwen3_5RMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.post_attention_layernorm = Qwen3_5RMSNorm(config.hidden_size, eps=config.rms_norm_eps)

    def forward(self, hidden_states: torch.Tensor, position_embeddings: Tuple[torch.Tensor, torch.Tensor],
                linear_mask: Optional[torch.Tensor] = None, full_attn_mask: Optional[torch.Tensor] = None,
                cache: Optional[Qwen3_5HybridCache] = None) -> torch.Tensor:
        hidden_states, pending = self.forward_pending(hidden_states, None, position_embeddings, linear_mask,
                                                      full_attn_mask, cache)
        return hidden_states + pending

    def forward_pending(self, hidden_states: torch.Tensor, pending: Optional[torch.Tensor],
                        position_embeddings: Tuple[torch.Tensor, torch.Tensor],
                        linear_mask: Optional[torch.Tensor] = None, full_attn_mask: Optional[torch.Tensor] = None,
                        cache: Optional[Qwen3_5HybridCache] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """The block with its last residual add left to the caller: takes the residual stream and the
        previous block's not yet added MLP output (or None) and returns the stream and this block's
        MLP output.  The add then runs inside the next norm's kernel (`add_forward`); the result is
        that of `forward` bit for bit (both round the sum to the activation dtype)."""
        if pending is None:
            h = self.input_layernorm(hidden_states)
        else:
            hidden_states, h = self.input_layernorm.add_forward(hidden_states, pending)
        if self.block_type == "linear_attention":
            h = self.linear_attn(h, attention_mask=linear_mask, cache=cache)
        else:
            h = self.self_attn(h, position_embeddings=position_embeddings, attention_mask=full_attn_mask, cache=cache)
        hidden_states, h = self.post_attention_layernorm.add_forward(hidden_states, h)  # residual + norm
        return hidden_states, self.mlp(h)


@dataclass
class Qwen3_5ModelOutput:
    """Output record with the reference's field names (config.py:146-151)."""
    last_hidden_state: torch.Tensor
    pooler_output: Optional[torch.Tensor] = None
    rope_deltas: Optional[torch.Tensor] = None
    past_key_values: Optional[Qwen3_5HybridCache] = None


class Qwen3_5TextModel(nn.Module):
    """Embedding, decoder layers, final norm (text.py:341-456), with the same position, mask and
    cache handling."""

    def __init__(self, config: Qwen3_5TextConfig):
        super().__init__()
        self.config = config
        pad = config.pad_token_id
        pad_idx = int(pad) if pad is not None and 0 <= int(pad) < int(config.vocab_size) else None
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_size, pad_idx)
        self.layers = nn.ModuleList([Qwen3_5DecoderLayer(config, i) for i in range(config.num_hidden_layers)])
        self.norm = Qwen3_5RMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.rotary_emb = Qwen3_5TextRotaryEmbedding(config)

    def forward(self, input_ids: Optional[torch.LongTensor] = None, attention_mask: Optional[torch.Tensor] = None,
                position_ids: Optional[torch.LongTensor] = None, inputs_embeds: Optional[torch.Tensor] = None,
                past_key_values: Optional[Qwen3_5HybridCache] = None, use_cache: bool = False,
                **kwargs) -> Qwen3_5ModelOutput:
        if (input_ids is None) ^ (inputs_embeds is not None):
            raise ValueError("Specify exactly one of input_ids or inputs_embeds.")
        if inputs_embeds is None:
            inputs_embeds = self.embed_tokens(input_ids)
        cache = past_key_values if past_key_values is not None else (Qwen3_5HybridCache() if use_cache else None)
        past = cache.past_seen_tokens if cache is not None else 0
        B, T, _ = inputs_embeds.shape
        dev = inputs_embeds.device
        if cache is not None and cache.record_checkpoints:
            cache.resolve_active_checkpoints(past, T)

        if position_ids is None:
            pos = torch.arange(past, past + T, device=dev).view(1, 1, -1)
            if cache is not None and cache.rope_deltas is not None and past > 0:
                pos = pos + cache.rope_deltas.to(device=dev).unsqueeze(0)
            position_ids = pos.expand(3, B, -1)
        elif position_ids.ndim == 2:
            position_ids = position_ids[None].expand(3, B, -1)
        elif position_ids.ndim == 3 and position_ids.shape[0] == 4:
            position_ids = position_ids[1:]

        linear_mask = full_mask = None
        if attention_mask is not None and attention_mask.ndim == 2 and not attention_mask.bool().all():
            linear_mask = attention_mask[:, -T:].bool()
            total = past + T
            causal = torch.ones((T, total), dtype=torch.bool, device=dev).tril(diagonal=past)
            m2 = attention_mask.bool()
            m2 = m2[:, :total] if m2.shape[1] >= total else F.pad(m2, (total - m2.shape[1], 0), value=True)
            full_mask = causal[None, None] & m2[:, None, None, :]

        h = inputs_embeds
        pe = self.rotary_emb(h, position_ids)
        pending = None  # each block's MLP output is added inside the next norm's kernel
        for layer in self.layers:
            h, pending = layer.forward_pending(h, pending, pe, linear_mask, full_mask, cache)
        if cache is not None:
            cache.past_seen_tokens = past + T
        out = self.norm(h) if pending is None else self.norm.add_forward(h, pending)[1]
        return Qwen3_5ModelOutput(last_hidden_state=out, past_key_values=cache)


class StackDecodeGraph:
    """Single-token decode steps of a `Qwen3_5TextModel` replayed from one CUDA graph.

    Built after a prefill into `cache` with `cache.kv_capacity` >= the final length.  The token of
    step i is column `cache.past_seen_tokens` of `ids` ([B, N] int64 on the device), its position
    that same column: both are read on the device, so the graph is position independent.  The
    attention layers switch to their static-KV path (write at the position, attend over the keys
    up to it); every DeltaNet layer's recurrent state is updated in place and its new conv state
    is copied back into the buffer the next step reads.  The first step runs eagerly (it also
    warms the libraries up), the graph is captured after it.  `step()` returns the step's final
    hidden state [B, 1, hidden] (a buffer the next step overwrites).
    """

    def __init__(self, model: Qwen3_5TextModel, cache: Qwen3_5HybridCache, ids: torch.Tensor):
        self.model, self.cache, self.ids = model, cache, ids
        dev = ids.device
        self.pos = torch.full((1,), int(cache.past_seen_tokens), dtype=torch.long, device=dev)
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.out: Optional[torch.Tensor] = None
        self._lin = [i for i, t in enumerate(model.config.layer_types) if t == "linear_attention"]
        bufs = getattr(cache, "_kv_buffers", {})
        for i, t in enumerate(model.config.layer_types):
            if t == "full_attention" and (i not in bufs or cache.key_cache.get(i) is None or
                                          cache.key_cache[i].data_ptr() != bufs[i][0].data_ptr()):
                raise ValueError("prefill the cache with kv_capacity set before building the decode graph")
        self._conv = {l: cache.conv_states[l] for l in self._lin}
        self.capacity = min(bufs[i][0].shape[2] for i in bufs) if bufs else 1 << 30

    def _one(self) -> torch.Tensor:
        B = self.ids.shape[0]
        tok = self.ids.gather(1, self.pos.view(1, 1).expand(B, 1))
        pid = self.pos.view(1, 1, 1).expand(3, B, 1)
        self.cache.static_pos = self.pos
        try:
            h = self.model(input_ids=tok, position_ids=pid, past_key_values=self.cache, use_cache=True)
        finally:
            self.cache.static_pos = None
        for l in self._lin:
            self._conv[l].copy_(self.cache.conv_states[l])
            self.cache.conv_states[l] = self._conv[l]
        self.pos.add_(1)
        return h.last_hidden_state

    def step(self) -> torch.Tensor:
        seen = int(self.cache.past_seen_tokens)
        if seen >= self.capacity:
            raise ValueError("the KV buffers are full")
        if self.graph is None:
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):  # the eager step doubles as the libraries' warm-up
                first = self._one()
            torch.cuda.current_stream().wait_stream(side)
            torch.cuda.synchronize()
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):  # recorded, not run: the output buffer fills on replay
                self.out = self._one()
            self.cache.past_seen_tokens = seen + 1
            return first
        self.graph.replay()
        self.cache.past_seen_tokens = seen + 1
        return self.out

    def finish(self) -> None:
        """Leave the cache as the eager path would: key / value entries trimmed to the tokens seen."""
        n = int(self.cache.past_seen_tokens)
        for i, (kb, vb) in getattr(self.cache, "_kv_buffers", {}).items():
            self.cache.key_cache[i] = kb[:, :, :n]
            self.cache.value_cache[i] = vb[:, :, :n]
        self.graph = None
