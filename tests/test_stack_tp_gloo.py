"""Tensor-parallel sharding of the decoder stack, host side, on CPU ranks over gloo.

The DeltaNet layers' sharding is covered by test_sharding_gloo.py (their token mixer needs the
GPU); here a stack of gated-attention layers and MLPs in fp32 is cut with ``shard_stack`` on 2 and
4 ranks (4 ranks put 1 query head per rank and a KV head on two ranks) and must give the
unsharded stack's hidden states for a prefill and a decode step after it, with each rank's KV
cache the slice of the unsharded one for the KV heads its queries read.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from visionstack_b200 import Qwen3_5HybridCache, Qwen3_5TextConfig
from visionstack_b200.stack import Qwen3_5TextModel
from visionstack_b200.stack_tp import attention_head_ranges, shard_stack

CFG = dict(vocab_size=97, hidden_size=64, intermediate_size=96, num_hidden_layers=2, num_attention_heads=4,
           num_key_value_heads=2, head_dim=16, layer_types=["full_attention", "full_attention"],
           pad_token_id=None, eos_token_id=None)


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _model() -> Qwen3_5TextModel:
    torch.manual_seed(11)
    m = Qwen3_5TextModel(Qwen3_5TextConfig(**CFG))
    with torch.no_grad():
        for name, p in m.named_parameters():
            p.normal_(0.0, 0.1 if "norm" in name else p.shape[-1] ** -0.5)
    return m.eval()


def _run(m, ids, tok):
    cache = Qwen3_5HybridCache()
    with torch.no_grad():
        h = m(input_ids=ids, past_key_values=cache, use_cache=True).last_hidden_state
        hd = m(input_ids=tok, past_key_values=cache, use_cache=True).last_hidden_state
    return h, hd, cache


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(5)
        ids = torch.randint(0, CFG["vocab_size"], (2, 13), generator=g)
        tok = torch.randint(0, CFG["vocab_size"], (2, 1), generator=g)
        ref = _model()
        h_ref, hd_ref, c_ref = _run(ref, ids, tok)
        m = shard_stack(_model(), rank, world)
        h, hd, c = _run(m, ids, tok)
        _, _, kv0, kv1 = attention_head_ranges(CFG["num_attention_heads"], CFG["num_key_value_heads"], rank, world)
        kv_err = max(max(float((c.key_cache[i] - c_ref.key_cache[i][:, kv0:kv1]).abs().max()),
                         float((c.value_cache[i] - c_ref.value_cache[i][:, kv0:kv1]).abs().max()))
                     for i in range(CFG["num_hidden_layers"]))
        q.put((rank, float((h - h_ref).abs().max()), float((hd - hd_ref).abs().max()), kv_err))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_stack_matches_unsharded(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # fp32 throughout; the sharded GEMMs and the all-reduce only reorder the sums
    for rank, e_pre, e_dec, kv_err in res:
        assert e_pre < 1e-5 and e_dec < 1e-5, f"rank {rank}: prefill err {e_pre}, decode err {e_dec}"
        assert kv_err < 1e-5, f"rank {rank}: KV cache differs from the slice of its KV heads by {kv_err}"


def test_attention_head_ranges():
    # 16 query / 2 KV heads (the stack workload): 8 ranks -> 2 query heads each, KV head r // 4
    assert [attention_head_ranges(16, 2, r, 8) for r in (0, 3, 4, 7)] == \
        [(0, 2, 0, 1), (6, 8, 0, 1), (8, 10, 1, 2), (14, 16, 1, 2)]
    assert attention_head_ranges(16, 2, 1, 2) == (8, 16, 1, 2)
    assert attention_head_ranges(16, 2, 0, 1) == (0, 16, 0, 2)
    with pytest.raises(ValueError):
        attention_head_ranges(12, 4, 1, 6)  # a rank's two queries would read two KV heads
    with pytest.raises(ValueError):
        attention_head_ranges(16, 2, 0, 3)
