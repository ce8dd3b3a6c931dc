"""Configuration and small modules the DeltaNet layer is built from.

``Qwen3_5TextConfig`` keeps the field names and defaults of the reference's
text config (ShadowBoxer/models/qwen35/config.py:184-254) so that a config
built for the reference constructs this layer unchanged; only the DeltaNet
fields are read here.  ``Qwen3_5RMSNormGated`` keeps the parameter name
``weight`` of config.py:130-134 for state-dict compatibility; inside the
layer its math runs in the token-mixer kernels' epilogue, and its
``forward(hidden_states, gate)`` runs the stand-alone ``gdn_rms_norm_gated``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional

import torch
import torch.nn.functional as F
from torch import nn

_FP8_DTYPES = {
    dt for dt in (getattr(torch, n, None) for n in (
        "float8_e4m3fn", "float8_e4m3fnuz", "float8_e5m2", "float8_e5m2fnuz", "float8_e8m0fnu"))
    if dt is not None
}


@dataclass
class Qwen3_5TextConfig:
    vocab_size: int = 248320
    hidden_size: int = 4096
    intermediate_size: int = 12288
    num_hidden_layers: int = 32
    num_attention_heads: int = 16
    num_key_value_heads: int = 4
    hidden_act: str = "silu"
    max_position_embeddings: int = 262144
    initializer_range: float = 0.02
    rms_norm_eps: float = 1e-6
    use_cache: bool = True
    tie_word_embeddings: bool = False
    attention_bias: bool = False
    attention_dropout: float = 0.0
    head_dim: int = 256
    linear_conv_kernel_dim: int = 4
    linear_key_head_dim: int = 128
    linear_value_head_dim: int = 128
    linear_num_key_heads: int = 16
    linear_num_value_heads: int = 32
    mtp_num_hidden_layers: int = 1
    layer_types: Optional[List[str]] = None
    pad_token_id: Optional[int] = 248044
    bos_token_id: Optional[int] = None
    eos_token_id: Optional[int] = 248044
    rope_parameters: Dict[str, Any] = field(default_factory=lambda: {
        "rope_type": "default", "rope_theta": 10000000.0, "partial_rotary_factor": 0.25,
        "mrope_section": [11, 11, 10]})

    def __post_init__(self) -> None:
        # every 4th layer is full attention, the rest linear attention
        if self.layer_types is None:
            self.layer_types = ["full_attention" if (i + 1) % 4 == 0 else "linear_attention"
                                for i in range(self.num_hidden_layers)]
        for name in ("pad_token_id", "eos_token_id"):
            v = getattr(self, name)
            if v is not None and not 0 <= int(v) < int(self.vocab_size):
                setattr(self, name, None)

    @classmethod
    def from_dict(cls, data: Dict[str, Any]) -> "Qwen3_5TextConfig":
        known = set(cls.__dataclass_fields__)
        return cls(**{k: v for k, v in data.items() if k in known})


def _linear(layer: nn.Linear, x: torch.Tensor) -> torch.Tensor:
    """Projection with the reference's dtype rules (config.py:55-68): fp8
    weights are upcast to the activation dtype, otherwise x is cast to the
    weight dtype."""
    w = layer.weight
    if w.dtype in _FP8_DTYPES:
        cdt = x.dtype if x.dtype in (torch.bfloat16, torch.float16, torch.float32) else torch.bfloat16
        b = layer.bias.to(cdt) if layer.bias is not None else None
        return F.linear(x.to(cdt), w.to(cdt), b)
    if x.dtype != w.dtype:
        x = x.to(w.dtype)
    return layer(x)


class Qwen3_5RMSNormGated(nn.Module):
    """Gated RMSNorm over the last dimension (config.py:130-143).  Inside the
    DeltaNet layer the normalisation is fused into the token-mixer kernels;
    ``forward`` is the stand-alone form for other callers and runs
    ``gdn_rms_norm_gated`` (CUDA tensors only, no CPU path)."""

    def __init__(self, hidden_size: int, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size))
        self.variance_epsilon = eps

    def forward(self, hidden_states: torch.Tensor, gate: torch.Tensor) -> torch.Tensor:
        from . import _lib
        codes = {torch.float32: _lib.GDN_DTYPE_F32, torch.bfloat16: _lib.GDN_DTYPE_BF16}
        for t in (hidden_states, gate, self.weight):
            if not t.is_cuda:
                raise RuntimeError("Qwen3_5RMSNormGated needs CUDA tensors (there is no CPU path)")
            if t.dtype not in codes:
                raise TypeError(f"unsupported dtype {t.dtype} (float32 or bfloat16)")
        dim = hidden_states.shape[-1]
        if gate.shape != hidden_states.shape or self.weight.shape != (dim,):
            raise ValueError(f"shapes {tuple(hidden_states.shape)}, gate {tuple(gate.shape)}, "
                             f"weight {tuple(self.weight.shape)} do not match")
        x = hidden_states.contiguous()
        gt = gate.contiguous()
        w = self.weight.detach().contiguous()
        out = torch.empty_like(x)
        rows = x.numel() // max(1, dim)
        if rows == 0:
            return out
        lib = _lib.load()
        with torch.cuda.device(x.device):
            _lib.check("gdn_rms_norm_gated", lib.gdn_rms_norm_gated(
                x.data_ptr(), gt.data_ptr(), w.data_ptr(), out.data_ptr(), rows, dim,
                float(self.variance_epsilon), codes[x.dtype], codes[gt.dtype], codes[w.dtype],
                torch.cuda.current_stream(x.device).cuda_stream))
        return out


def q_scale(head_k_dim: int) -> float:
    return float(math.pow(head_k_dim, -0.5))
