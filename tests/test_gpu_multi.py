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


def _mixer_worker(rank, world, port, q):
    """Every rank gets the same full projection outputs (seeded numpy), slices its heads' channels,
    runs the token mixer on its shard and returns its outputs and states; then its out_proj partial
    is all-reduced."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import torch.nn.functional as F

        from tests.test_gpu_mixer import mixer_inputs
        from visionstack_b200.sharding import HeadShardedGatedDeltaNet, shard_ranges
        dev = torch.device("cuda", rank)
        full = W.make_layer_params(SHAPE, 3, "bf16")
        layer = HeadShardedGatedDeltaNet(full, SHAPE, 0, rank, world, device=dev, dtype=torch.bfloat16).layer
        r = shard_ranges(SHAPE, rank, world)
        d = mixer_inputs(SHAPE, 2, 200, "bf16", seed=91, with_state=True)
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev).to(torch.bfloat16)  # noqa: E731
        cols = np.concatenate([np.arange(*r["q"]), np.arange(*r["k"]), np.arange(*r["v"])])
        h0, h1 = r["heads"]
        c0, c1 = r["vcols"]
        mixed = t(d["mixed"][..., cols])
        z, a, b = t(d["z"][..., c0:c1]), t(d["a"][..., h0:h1]), t(d["b"][..., h0:h1])
        cs = t(d["conv_state"][:, cols])
        S0 = torch.from_numpy(d["rec_state"][:, h0:h1]).to(dev)
        S = torch.empty_like(S0)
        cs_out = torch.empty_like(cs)
        with torch.no_grad():
            core = layer.mixer(mixed, z, b, a, conv_state=cs, rec_state=S0, conv_state_out=cs_out, rec_state_out=S,
                               token_by_token=False)
            y = F.linear(core, layer.out_proj.weight)
        dist.all_reduce(y, op=dist.ReduceOp.SUM)
        torch.cuda.synchronize()
        outs = [torch.empty_like(core) for _ in range(world)]
        states = [torch.empty_like(S) for _ in range(world)]
        dist.all_gather(outs, core)
        dist.all_gather(states, S)
        if rank == 0:
            q.put((torch.cat(outs, -1).float().cpu().numpy(), torch.cat(states, 1).cpu().numpy(),
                   y.float().cpu().numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_sharded_mixer_matches_oracle():
    """With identical projection outputs on every rank the sharded token mixer is held to the flat
    tolerances against the oracle (outputs 2e-2, state 1e-3); the all-reduced out_proj equals one
    GEMM over the gathered outputs up to the rounding of the bf16 partial sums."""
    from oracle import gdn_oracle as O
    from tests.helpers import assert_bf16_close, assert_state_close
    from tests.test_gpu_mixer import mixer_inputs
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_mixer_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    core, states, y = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    full = W.make_layer_params(SHAPE, 3, "bf16")
    d = mixer_inputs(SHAPE, 2, 200, "bf16", seed=91, with_state=True)
    r_out, _, r_S, _, _ = O.mixer_forward(SHAPE, d["mixed"], d["z"].reshape(2, 200, SHAPE.num_v_heads,
                                                                               SHAPE.head_v_dim),
                                          d["a"], d["b"], full["conv1d.weight"], full["A_log"], full["dt_bias"],
                                          full["norm.weight"], "bf16", d["conv_state"], d["rec_state"], chunk=True)
    assert_bf16_close(core, r_out, "sharded mixer outputs (2 GPUs)")
    assert_state_close(states, r_S, "sharded mixer final state (2 GPUs)")
    ry = O.cast(np.matmul(core, full["out_proj.weight"].T.astype(np.float32)), "bf16")
    assert_bf16_close(y, ry, "all-reduced out_proj partials", scale=2.0)
