"""Value-head sharding of the DeltaNet layer across the GPUs of one node.

Each (batch row, value head) recurrence is independent, and value head h
reads key head h // (Hv / Hk).  Rank r of N therefore owns value heads
[r*Hv/N, (r+1)*Hv/N) and exactly the key heads [r*Hk/N, (r+1)*Hk/N) they
read, so the token mixer runs with no communication.  The only exchange is
the sum of the row-parallel ``out_proj`` partial outputs: one NCCL
all-reduce (bf16, sum) of [B, T, hidden] per layer.

Parameter partitioning (reference parameter names, deltanet.py:425-445):
``in_proj_qkv`` / ``conv1d.weight``: the q, k and v channel ranges of the
shard (three row ranges); ``in_proj_z``, ``in_proj_a``, ``in_proj_b``,
``A_log``, ``dt_bias``: the value-head range; ``norm.weight``: replicated;
``out_proj``: the value-head column range.  Caches hold each rank's own
conv-state channels and recurrent-state heads.
"""
from __future__ import annotations

from dataclasses import replace
from typing import Dict, Optional, Tuple

import numpy as np

from .workloads import LayerShape


def shard_ranges(shape: LayerShape, rank: int, world: int):
    if shape.num_v_heads % world or shape.num_k_heads % world:
        raise ValueError(f"{world} ranks do not divide {shape.num_k_heads} key / {shape.num_v_heads} value heads")
    hk, hv = shape.num_k_heads // world, shape.num_v_heads // world
    dk, dv = shape.head_k_dim, shape.head_v_dim
    k0, v0 = rank * hk, rank * hv
    kd = shape.key_dim
    q_rows = (k0 * dk, (k0 + hk) * dk)
    k_rows = (kd + k0 * dk, kd + (k0 + hk) * dk)
    v_rows = (2 * kd + v0 * dv, 2 * kd + (v0 + hv) * dv)
    return {"q": q_rows, "k": k_rows, "v": v_rows, "heads": (v0, v0 + hv), "vcols": (v0 * dv, (v0 + hv) * dv),
            "local": replace(shape, num_k_heads=hk, num_v_heads=hv)}


def _rows(a, r):
    return a[r[0]:r[1]]


def shard_params(params: Dict[str, "np.ndarray"], shape: LayerShape, rank: int, world: int
                 ) -> Tuple[Dict[str, "np.ndarray"], LayerShape]:
    """Slice a full state dict (numpy or torch tensors) for ``rank``."""
    r = shard_ranges(shape, rank, world)
    cat = (lambda xs: np.concatenate(xs, 0)) if isinstance(params["A_log"], np.ndarray) else _torch_cat
    out = dict(params)
    qkv = params["in_proj_qkv.weight"]
    out["in_proj_qkv.weight"] = cat([_rows(qkv, r["q"]), _rows(qkv, r["k"]), _rows(qkv, r["v"])])
    cw = params["conv1d.weight"]
    out["conv1d.weight"] = cat([_rows(cw, r["q"]), _rows(cw, r["k"]), _rows(cw, r["v"])])
    out["in_proj_z.weight"] = _rows(params["in_proj_z.weight"], r["vcols"])
    for name in ("in_proj_a.weight", "in_proj_b.weight", "A_log", "dt_bias"):
        out[name] = _rows(params[name], r["heads"])
    c0, c1 = r["vcols"]
    out["out_proj.weight"] = params["out_proj.weight"][:, c0:c1]
    out["norm.weight"] = params["norm.weight"]
    return {k: (v.copy() if isinstance(v, np.ndarray) else v.clone().contiguous()) for k, v in out.items()}, \
        r["local"]


def _torch_cat(xs):
    import torch
    return torch.cat(xs, 0)


class HeadShardedGatedDeltaNet:
    """The DeltaNet layer on one rank of a value-head-sharded group.

    ``forward`` runs the rank's projections, the fused token mixer on its
    heads, its slice of ``out_proj``, and one all-reduce (sum) of the partial
    outputs over ``group`` (NCCL on GPUs, or the one-shot peer all-reduce of
    ``peer`` where the output fits it).  The cache passed in holds this
    rank's shard of the states.
    """

    def __init__(self, full_state_dict, shape: LayerShape, layer_idx: int, rank: int, world: int,
                 group=None, device=None, dtype=None, peer=None):
        import torch

        from .config import Qwen3_5TextConfig
        from .deltanet import Qwen3_5GatedDeltaNet
        params, local = shard_params(full_state_dict, shape, rank, world)
        cfg = Qwen3_5TextConfig(hidden_size=shape.hidden_size, linear_num_key_heads=local.num_k_heads,
                                linear_num_value_heads=local.num_v_heads, linear_key_head_dim=shape.head_k_dim,
                                linear_value_head_dim=shape.head_v_dim, linear_conv_kernel_dim=shape.conv_kernel,
                                rms_norm_eps=shape.rms_norm_eps)
        self.layer = Qwen3_5GatedDeltaNet(cfg, layer_idx)
        with torch.no_grad():
            for name, p in self.layer.named_parameters():
                t = params[name]
                t = torch.from_numpy(t) if isinstance(t, np.ndarray) else t
                if name not in ("A_log", "dt_bias") and dtype is not None:
                    t = t.to(dtype)
                p.data = t
        if device is not None:
            self.layer.to(device)
        self.local_shape = local
        self.group = group
        self.world = world
        self.peer = peer  # optional peer.PeerAllReduce: the one-shot NVLink sum for decode-sized outputs

    def __call__(self, hidden_states, attention_mask=None, cache=None, async_op: bool = False):
        import torch.distributed as dist
        partial = self.layer(hidden_states, attention_mask=attention_mask, cache=cache)
        if self.world > 1 and not async_op and self.peer is not None and self.peer.fits(partial):
            return self.peer(partial)
        if self.world > 1:
            work = dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=self.group, async_op=async_op)
            if async_op:
                return partial, work
        return partial


__all__ = ["shard_ranges", "shard_params", "HeadShardedGatedDeltaNet"]
