"""Value-head sharding across GPUs with NCCL (skipped with fewer than 2 GPUs).

Each rank runs its shard of the layer (its key/value heads, its out_proj
columns) and one all-reduce sums the partial outputs; the result must match
the unsharded layer, and the ranks' state shards must be the head slices of
the unsharded state.
"""
from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from visionstack_b200 import workloads as W

pytestmark = pytest.mark.gpu

SHAPE = W.LayerShape(512, 4, 8, 128, 128)


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from visionstack_b200 import Qwen3_5HybridCache
        from visionstack_b200.sharding import HeadShardedGatedDeltaNet
        full = W.make_layer_params(SHAPE, 3, "bf16")
        layer = HeadShardedGatedDeltaNet(full, SHAPE, 0, rank, world, device=torch.device("cuda", rank),
                                         dtype=torch.bfloat16)
        wl = W.Workload("mg", SHAPE, 2, 96, 1, "bf16", 4, 3)
        x = torch.from_numpy(W.make_hidden(wl)).cuda().to(torch.bfloat16)
        xd = torch.from_numpy(W.make_hidden(wl, seq_len=1, seed_offset=1)).cuda().to(torch.bfloat16)
        with torch.inference_mode():
            cache = Qwen3_5HybridCache()
            y = layer(x, cache=cache)
            cache.past_seen_tokens = 96
            yd = layer(xd, cache=cache)
            states = [torch.empty_like(cache.recurrent_states[0]) for _ in range(world)]
            dist.all_gather(states, cache.recurrent_states[0])
        torch.cuda.synchronize()
        if rank == 0:
            q.put((y.float().cpu().numpy(), yd.float().cpu().numpy(), torch.cat(states, 1).cpu().numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_head_sharded_layer_matches_unsharded():
    from tests.helpers import assert_bf16_close, assert_state_close
    from tests.test_gpu_mixer import make_layer
    from visionstack_b200 import Qwen3_5HybridCache
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    y, yd, states = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    m, _ = make_layer(SHAPE, "bf16", seed=3)
    wl = W.Workload("mg", SHAPE, 2, 96, 1, "bf16", 4, 3)
    x = torch.from_numpy(W.make_hidden(wl)).cuda().to(torch.bfloat16)
    xd = torch.from_numpy(W.make_hidden(wl, seq_len=1, seed_offset=1)).cuda().to(torch.bfloat16)
    with torch.inference_mode():
        cache = Qwen3_5HybridCache()
        ry = m(x, cache=cache)
        cache.past_seen_tokens = 96
        ryd = m(xd, cache=cache)
    # The sharded sum adds the out_proj partials in another order, and each
    # rank's projection is a different (narrower) GEMM whose bf16 outputs may
    # differ from the full GEMM's in the last bit: outputs get two roundings of
    # slack, and the states (which accumulate those inputs) 5e-3.
    assert_bf16_close(y, ry, "sharded prefill", scale=2.0)
    assert_bf16_close(yd, ryd, "sharded decode", scale=2.0)
    assert_state_close(states, cache.recurrent_states[0], "sharded state", scale=5.0)
    assert np.isfinite(y).all()
