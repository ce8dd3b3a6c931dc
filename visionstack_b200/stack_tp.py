"""Tensor-parallel sharding of the hybrid decoder stack over the GPUs of one node.

The stack workload shards the DeltaNet value heads over 1 / 2 / 4 / 8 GPUs; every other part of
a layer is cut to match, so that each rank does 1/N of every layer's work and a layer exchanges
one all-reduce per sub-block (two per layer):

* Gated DeltaNet (deltanet.py:410-563): value heads [r Hv/N, (r+1) Hv/N) and exactly the key
  heads they read (``sharding.shard_params``), ``out_proj`` column slice; the partial outputs
  are summed.
* Gated attention (text.py:89-212): query heads [r H/N, (r+1) H/N) (their query and gate rows of
  ``q_proj``) and the key / value heads those queries read (query head h reads KV head
  h // (H / KVH); with more ranks than KV heads, a KV head is held by every rank whose queries
  read it), ``o_proj`` column slice (its bias, if any, on rank 0 only); summed.
* MLP (text.py:215-230): ``gate_proj`` / ``up_proj`` rows [r I/N, (r+1) I/N), ``down_proj``
  column slice; summed.
* Embedding, RMSNorms and the rotary embedding: replicated.

Each sum is an all-reduce of the sub-block's [B, T, hidden] output in place, run by a forward
hook (with a ``peer.PeerAllReduce`` the decode-sized ones take its one-shot NVLink kernel, the
rest the process group's all-reduce, NCCL on GPUs), so every shard keeps the reference's
parameter names (with local shapes) and the decoder layer, the cache and ``StackDecodeGraph``
work unchanged (a captured decode step holds the all-reduces).  Caches hold each rank's own states: its DeltaNet heads and its KV heads.
The reference has no tensor parallelism; this is the multi-GPU form of its stack.
"""
from __future__ import annotations

from dataclasses import replace
from typing import Optional

import torch
import torch.distributed as dist
from torch import nn

from .deltanet import Qwen3_5GatedDeltaNet
from .sharding import shard_params
from .workloads import LayerShape


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def attention_head_ranges(num_heads: int, num_kv_heads: int, rank: int, world: int):
    """Query heads [h0, h1) of ``rank`` and the KV heads [kv0, kv1) they read."""
    _check(num_heads % world == 0, f"{world} ranks do not divide {num_heads} attention heads")
    _check(num_heads % num_kv_heads == 0, "query heads must be a multiple of the KV heads")
    per = num_heads // world
    groups = num_heads // num_kv_heads
    h0, h1 = rank * per, (rank + 1) * per
    kv0, kv1 = h0 // groups, (h1 - 1) // groups + 1
    _check(per % (kv1 - kv0) == 0 and (per // (kv1 - kv0) == groups or kv1 - kv0 == 1),
           f"{world} ranks do not split {num_heads} query / {num_kv_heads} KV heads into whole groups")
    return h0, h1, kv0, kv1


def _sum_hook(group, peer):
    from .peer import sum_partials

    def hook(module, args, output):
        return sum_partials(output, peer, group)
    return hook


def _assign(module: nn.Module, tensors) -> None:
    with torch.no_grad():
        for name, p in module.named_parameters():
            p.data = tensors[name].contiguous()


def _shard_deltanet(old: Qwen3_5GatedDeltaNet, cfg, idx: int, rank: int, world: int) -> Qwen3_5GatedDeltaNet:
    shape = LayerShape(cfg.hidden_size, cfg.linear_num_key_heads, cfg.linear_num_value_heads,
                       cfg.linear_key_head_dim, cfg.linear_value_head_dim, cfg.linear_conv_kernel_dim,
                       cfg.rms_norm_eps)
    full = {k: v.detach() for k, v in old.state_dict().items()}
    params, local = shard_params(full, shape, rank, world)
    new = Qwen3_5GatedDeltaNet(replace(cfg, linear_num_key_heads=local.num_k_heads,
                                       linear_num_value_heads=local.num_v_heads), idx)
    _assign(new, params)
    new.inplace_state, new.fuse_in_proj = old.inplace_state, old.fuse_in_proj
    return new


def _shard_attention(old: nn.Module, cfg, idx: int, rank: int, world: int) -> nn.Module:
    from .stack import Qwen3_5Attention
    hd = old.head_dim
    h0, h1, kv0, kv1 = attention_head_ranges(old.num_heads, old.num_kv_heads, rank, world)
    new = Qwen3_5Attention(replace(cfg, num_attention_heads=h1 - h0, num_key_value_heads=kv1 - kv0,
                                   head_dim=hd), idx)
    sd = {k: v.detach() for k, v in old.state_dict().items()}
    t = {
        "q_proj.weight": sd["q_proj.weight"][2 * hd * h0:2 * hd * h1],
        "k_proj.weight": sd["k_proj.weight"][hd * kv0:hd * kv1],
        "v_proj.weight": sd["v_proj.weight"][hd * kv0:hd * kv1],
        "o_proj.weight": sd["o_proj.weight"][:, hd * h0:hd * h1],
        "q_norm.weight": sd["q_norm.weight"],
        "k_norm.weight": sd["k_norm.weight"],
    }
    if "q_proj.bias" in sd:
        t["q_proj.bias"] = sd["q_proj.bias"][2 * hd * h0:2 * hd * h1]
        t["k_proj.bias"] = sd["k_proj.bias"][hd * kv0:hd * kv1]
        t["v_proj.bias"] = sd["v_proj.bias"][hd * kv0:hd * kv1]
        t["o_proj.bias"] = sd["o_proj.bias"] if rank == 0 else torch.zeros_like(sd["o_proj.bias"])
    _assign(new, t)
    return new


def _shard_mlp(old: nn.Module, cfg, rank: int, world: int) -> nn.Module:
    from .stack import Qwen3_5MLP
    inter = old.gate_proj.weight.shape[0]
    _check(inter % world == 0, f"{world} ranks do not divide the MLP width {inter}")
    per = inter // world
    r0, r1 = rank * per, (rank + 1) * per
    new = Qwen3_5MLP(cfg, per)
    sd = {k: v.detach() for k, v in old.state_dict().items()}
    _assign(new, {"gate_proj.weight": sd["gate_proj.weight"][r0:r1], "up_proj.weight": sd["up_proj.weight"][r0:r1],
                  "down_proj.weight": sd["down_proj.weight"][:, r0:r1]})
    return new


def shard_stack(model: nn.Module, rank: int, world: int, group: Optional[object] = None,
                peer: Optional[object] = None) -> nn.Module:
    """Cut a loaded ``Qwen3_5TextModel`` down to ``rank``'s shard of a ``world``-way tensor-parallel
    group, in place, and attach the all-reduces (``peer``: an optional ``PeerAllReduce`` of the
    group for the outputs that fit it); returns the model.  Every rank passes the same full
    weights.  With ``world`` = 1 the model is returned unchanged."""
    if world == 1:
        return model
    cfg = model.config
    hook = _sum_hook(group, peer)
    for idx, layer in enumerate(model.layers):
        if layer.block_type == "linear_attention":
            layer.linear_attn = _shard_deltanet(layer.linear_attn, cfg, idx, rank, world)
            layer.linear_attn.register_forward_hook(hook)
        else:
            layer.self_attn = _shard_attention(layer.self_attn, cfg, idx, rank, world)
            layer.self_attn.register_forward_hook(hook)
        layer.mlp = _shard_mlp(layer.mlp, cfg, rank, world)
        layer.mlp.register_forward_hook(hook)
    model.tp_rank, model.tp_world = rank, world
    return model


__all__ = ["attention_head_ranges", "shard_stack"]
