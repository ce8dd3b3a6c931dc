"""Value-head sharding, host side, on 2 CPU ranks over gloo.

Each rank slices the full state dict with ``shard_params``, runs its shard
of the layer (the numpy oracle stands in for the GPU mixer here), and the
row-parallel out_proj partials are summed with an all-reduce.  The result
must equal the unsharded layer, and the per-rank states must be the head
slices of the unsharded states.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import gdn_oracle as O
from visionstack_b200 import workloads as W
from visionstack_b200.sharding import shard_params, shard_ranges

SHAPE = W.LayerShape(128, 2, 4, 32, 32)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = W.make_layer_params(SHAPE, 5, "f32")
        local, lshape = shard_params(full, SHAPE, rank, world)
        x = W.make_hidden(W.Workload("g", SHAPE, 2, 40, 1, "f32", 9, 5))
        cache = O.OracleCache()
        part = O.deltanet_layer_forward(local, lshape, x, "f32", cache=cache)
        t = torch.from_numpy(part.copy())
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        states = [torch.zeros(2, lshape.num_v_heads, 32, 32) for _ in range(world)]
        dist.all_gather(states, torch.from_numpy(cache.recurrent_states[0].copy()))
        if rank == 0:
            q.put((t.numpy(), torch.cat(states, 1).numpy(), cache.conv_states[0].shape))
    finally:
        dist.destroy_process_group()


def test_shard_ranges_cover_every_channel_once():
    for world in (1, 2):
        seen = []
        for r in range(world):
            rg = shard_ranges(SHAPE, r, world)
            for key in ("q", "k", "v"):
                seen.extend(range(*rg[key]))
        assert sorted(seen) == list(range(SHAPE.conv_dim))


def test_qwen_shape_shards_on_8_ranks():
    for world in (1, 2, 4, 8):
        rg = shard_ranges(W.SHAPE_QWEN, world - 1, world)
        assert rg["local"].num_v_heads == 32 // world and rg["local"].num_k_heads == 16 // world
    with pytest.raises(ValueError):
        shard_ranges(W.SHAPE_QWEN, 0, 3)


def test_two_rank_sharded_layer_matches_unsharded():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    y, states, conv_shape = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    full = W.make_layer_params(SHAPE, 5, "f32")
    x = W.make_hidden(W.Workload("g", SHAPE, 2, 40, 1, "f32", 9, 5))
    cache = O.OracleCache()
    ref = O.deltanet_layer_forward(full, SHAPE, x, "f32", cache=cache)
    assert float(np.max(np.abs(y - ref))) < 1e-4
    assert float(np.max(np.abs(states - cache.recurrent_states[0]))) < 1e-5
    assert conv_shape == (2, SHAPE.conv_dim // world, 3)
