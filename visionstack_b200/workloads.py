"""Seeded synthetic workloads for the Gated DeltaNet token mixer.

The layer shapes and seeds are the five benchmark configurations of the
DeltaNet path (decoder layer ``Qwen3_5GatedDeltaNet``,
ShadowBoxer/models/qwen35/deltanet.py:410-563):

* ``cpu_plumbing``  B1  T256 (+16 decode)  hidden 1024, 8 k-heads / 8 v-heads, fp32
* ``decode``        B64 T1 x 512 steps     hidden 2048, 16 k-heads / 32 v-heads, bf16
* ``prefill``       B8  T8192              same heads as ``decode``, bf16
* ``rollback``      B16, 4-token drafts x 1024 steps, accept counts U{0..4}

There is no public dataset for this path, so every input is drawn from
``numpy.random.default_rng(seed)`` (PCG64, stable across machines and numpy
versions).  Weights are xavier-uniform with the fans torch assigns to each
parameter's own shape; the decay gate is realised at layer level as
``A_log := a ~ U(-1, 1)`` and ``dt_bias := 0`` so that
``g = -exp(A_log) * softplus(in_proj_a(x))`` keeps ``alpha = exp(g)`` in (0, 1].

This module is numpy-only: importing it never loads CUDA code.
"""
from __future__ import annotations

from dataclasses import dataclass, replace
from typing import Dict

import numpy as np


@dataclass(frozen=True)
class LayerShape:
    hidden_size: int
    num_k_heads: int
    num_v_heads: int
    head_k_dim: int
    head_v_dim: int
    conv_kernel: int = 4
    rms_norm_eps: float = 1e-6

    @property
    def key_dim(self) -> int:
        return self.num_k_heads * self.head_k_dim

    @property
    def value_dim(self) -> int:
        return self.num_v_heads * self.head_v_dim

    @property
    def conv_dim(self) -> int:
        return 2 * self.key_dim + self.value_dim


SHAPE_SMALL = LayerShape(1024, 8, 8, 128, 128)
SHAPE_QWEN = LayerShape(2048, 16, 32, 128, 128)
# The tiny hybrid text model the reference's own self-tests build
# (ShadowBoxer/sanitycheck/gate3_models.py:1016-1051): hidden 128, 2 k-heads,
# 4 v-heads, head dim 32.
SHAPE_TINY = LayerShape(128, 2, 4, 32, 32)


@dataclass(frozen=True)
class Workload:
    name: str
    shape: LayerShape
    batch: int
    seq_len: int
    steps: int
    dtype: str  # activation / parameter dtype: "f32" or "bf16"
    x_seed: int
    w_seed: int


WORKLOADS: Dict[str, Workload] = {
    "cpu_plumbing": Workload("cpu_plumbing", SHAPE_SMALL, 1, 256, 16, "f32", 0, 1),
    "decode": Workload("decode", SHAPE_QWEN, 64, 1, 512, "bf16", 2, 1),
    "prefill": Workload("prefill", SHAPE_QWEN, 8, 8192, 1, "bf16", 3, 1),
    "rollback": Workload("rollback", SHAPE_QWEN, 16, 4, 1024, "bf16", 5, 1),
}


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), kept as float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32)
    lsb = (u >> np.uint32(16)) & np.uint32(1)
    r = ((u + np.uint32(0x7FFF) + lsb) & np.uint32(0xFFFF0000)).view(np.float32)
    nan = np.isnan(x)
    if nan.any():
        r = np.where(nan, x, r)
    return r


def cast(x: np.ndarray, dtype: str) -> np.ndarray:
    """Represent ``x`` in ``dtype`` ("f32" or "bf16"); storage stays float32."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "bf16":
        return round_bf16(x)
    if dtype == "f32":
        return x
    raise ValueError(f"unsupported dtype {dtype!r}")


def _xavier(rng: np.random.Generator, shape, fan_in: int, fan_out: int) -> np.ndarray:
    bound = float(np.sqrt(6.0 / float(fan_in + fan_out)))
    return rng.uniform(-bound, bound, size=shape).astype(np.float32)


def make_layer_params(shape: LayerShape, seed: int, dtype: str) -> Dict[str, np.ndarray]:
    """State-dict arrays (reference parameter names, deltanet.py:425-445).

    ``A_log`` and ``dt_bias`` stay float32 whatever ``dtype`` is, as the
    reference loader keeps them (ShadowBoxer/core/loader.py:57-78).
    """
    rng = np.random.default_rng(seed)
    H, cd, vd, hv, K = shape.hidden_size, shape.conv_dim, shape.value_dim, shape.num_v_heads, shape.conv_kernel
    p = {
        "in_proj_qkv.weight": _xavier(rng, (cd, H), H, cd),
        "in_proj_z.weight": _xavier(rng, (vd, H), H, vd),
        "in_proj_b.weight": _xavier(rng, (hv, H), H, hv),
        "in_proj_a.weight": _xavier(rng, (hv, H), H, hv),
        # torch fans of a depthwise Conv1d weight [C, 1, K]: in = 1*K, out = C*K
        "conv1d.weight": _xavier(rng, (cd, 1, K), K, cd * K),
        "out_proj.weight": _xavier(rng, (H, vd), vd, H),
        "norm.weight": np.ones((shape.head_v_dim,), dtype=np.float32),
    }
    p = {k: cast(v, dtype) for k, v in p.items()}
    p["A_log"] = rng.uniform(-1.0, 1.0, size=(hv,)).astype(np.float32)
    p["dt_bias"] = np.zeros((hv,), dtype=np.float32)
    return p


def make_hidden(wl: Workload, seq_len: int | None = None, seed_offset: int = 0) -> np.ndarray:
    """x ~ N(0, 1) of shape [B, T, hidden] in the workload dtype."""
    T = wl.seq_len if seq_len is None else seq_len
    rng = np.random.default_rng(wl.x_seed + 1000003 * seed_offset)
    x = rng.standard_normal((wl.batch, T, wl.shape.hidden_size), dtype=np.float32)
    return cast(x, wl.dtype)


def make_decode_states(wl: Workload) -> Dict[str, np.ndarray]:
    """Pre-filled decode states: S0 ~ N(0, 0.02^2) fp32, conv state ~ N(0, 1)."""
    s = wl.shape
    rng = np.random.default_rng(wl.x_seed + 77)
    rec = (0.02 * rng.standard_normal(
        (wl.batch, s.num_v_heads, s.head_k_dim, s.head_v_dim), dtype=np.float32)).astype(np.float32)
    conv = cast(rng.standard_normal((wl.batch, s.conv_dim, s.conv_kernel - 1), dtype=np.float32), wl.dtype)
    return {"recurrent": rec, "conv": conv}


def make_gate_inputs(rng: np.random.Generator, B: int, T: int, H: int):
    """Kernel-level gates: beta = sigmoid(N(0,1)), g = -softplus(N(0,1)) * exp(a), a ~ U(-1,1) per head."""
    beta = 1.0 / (1.0 + np.exp(-rng.standard_normal((B, T, H)).astype(np.float32)))
    a = rng.uniform(-1.0, 1.0, size=(H,)).astype(np.float32)
    n = rng.standard_normal((B, T, H)).astype(np.float32)
    g = -np.log1p(np.exp(n)) * np.exp(a)[None, None, :]
    return g.astype(np.float32), beta.astype(np.float32)


def with_batch(wl: Workload, batch: int) -> Workload:
    return replace(wl, batch=batch)


# ---------------------------------------------------------------------------
# The hybrid decoder stack (ShadowBoxer/models/qwen35/text.py): every 4th layer
# full attention, the rest Gated DeltaNet.
# ---------------------------------------------------------------------------

# The 48-layer workload: hidden 2048, 16 query / 2 KV heads of 256, the DeltaNet heads of the
# decode / prefill workloads, vocab 151936; the MLP width is the reference config's default
# (12288), as the workload leaves it open.  B32, prefill 4096 tokens then 256 decode steps.
STACK_48 = dict(vocab_size=151936, hidden_size=2048, intermediate_size=12288, num_hidden_layers=48,
                num_attention_heads=16, num_key_value_heads=2, head_dim=256, linear_num_key_heads=16,
                linear_num_value_heads=32, linear_key_head_dim=128, linear_value_head_dim=128,
                linear_conv_kernel_dim=4, rms_norm_eps=1e-6)
STACK_48_RUN = dict(batch=32, prefill=4096, decode=256, seed=4)

# A 4-layer stack (3 DeltaNet + 1 attention) small enough for the reference on the host.
STACK_TINY = dict(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=4,
                  num_attention_heads=4, num_key_value_heads=2, head_dim=64, linear_num_key_heads=2,
                  linear_num_value_heads=4, linear_key_head_dim=64, linear_value_head_dim=64,
                  linear_conv_kernel_dim=4, rms_norm_eps=1e-6)


def make_stack_params(shapes: Dict[str, tuple], seed: int, dtype: str) -> Dict[str, np.ndarray]:
    """Seeded arrays for every entry of a stack's state dict, given its names and shapes.

    Each tensor draws from its own generator keyed by (seed, crc32 of its name), so the values do
    not depend on the order a model lists its parameters in.  Linear weights ~ N(0, 1/fan_in),
    embeddings ~ N(0, 1), zero-centred RMSNorm weights ~ N(0, 0.1^2), the gated norm's weight
    1 + N(0, 0.1^2), conv weights xavier-uniform, ``A_log`` ~ U(-1, 1) and ``dt_bias`` ~
    N(0, 0.1^2) (these two stay float32, as the reference loader keeps them).
    """
    import zlib
    out: Dict[str, np.ndarray] = {}
    for name in sorted(shapes):
        shp = tuple(int(s) for s in shapes[name])
        rng = np.random.default_rng([int(seed), zlib.crc32(name.encode())])
        if name.endswith("A_log"):
            out[name] = rng.uniform(-1.0, 1.0, size=shp).astype(np.float32)
            continue
        if name.endswith("dt_bias"):
            out[name] = (0.1 * rng.standard_normal(shp)).astype(np.float32)
            continue
        if name.endswith("linear_attn.norm.weight"):
            v = 1.0 + 0.1 * rng.standard_normal(shp)
        elif name.endswith("norm.weight") or name.endswith("layernorm.weight"):
            v = 0.1 * rng.standard_normal(shp)
        elif name.endswith("conv1d.weight"):
            v = _xavier(rng, shp, shp[2], shp[0] * shp[2])
        elif name.endswith("embed_tokens.weight"):
            v = rng.standard_normal(shp)
        elif len(shp) == 2:
            v = rng.standard_normal(shp) / np.sqrt(shp[1])
        else:
            v = 0.02 * rng.standard_normal(shp)
        out[name] = cast(np.asarray(v, dtype=np.float32), dtype)
    return out


def make_stack_calls(cfg: Dict, seed: int = 4):
    """Token ids and the call sequence of the small stack fixture: a 70-token prefill with a
    cache, three 1-token decode steps, one 4-token step, and separately a 40-token call without a
    cache under a 2-D attention mask with a hole (row 1, positions 10..12)."""
    rng = np.random.default_rng(seed)
    ids = rng.integers(0, cfg["vocab_size"], size=(2, 77), dtype=np.int64)
    spans = [(0, 70), (70, 71), (71, 72), (72, 73), (73, 77)]
    mask = np.ones((2, 40), dtype=np.int64)
    mask[1, 10:13] = 0
    return ids, spans, mask
