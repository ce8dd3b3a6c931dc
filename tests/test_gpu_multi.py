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


STACK_CFG = dict(vocab_size=256, hidden_size=512, intermediate_size=1024, num_hidden_layers=4, num_attention_heads=4,
                 num_key_value_heads=2, head_dim=128, linear_num_key_heads=4, linear_num_value_heads=8,
                 linear_key_head_dim=128, linear_value_head_dim=128, linear_conv_kernel_dim=4, rms_norm_eps=1e-6)


def _stack_model(dev):
    """4 layers (3 DeltaNet + 1 gated attention), seeded random bf16 weights, the same on every rank."""
    from visionstack_b200 import Qwen3_5TextConfig
    from visionstack_b200.stack import Qwen3_5TextModel
    cfg = Qwen3_5TextConfig(**STACK_CFG)
    with torch.device("meta"):
        m = Qwen3_5TextModel(cfg)
    m = m.to_empty(device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(17)
    with torch.no_grad():
        for name, p in m.named_parameters():
            if name.endswith("A_log"):
                p.data = torch.empty(p.shape, device=dev).uniform_(-1.0, 1.0, generator=g)
            elif name.endswith("dt_bias"):
                p.data = torch.zeros(p.shape, device=dev)
            elif name.endswith("linear_attn.norm.weight"):
                p.data = torch.ones(p.shape, device=dev, dtype=torch.bfloat16)
            elif "norm" in name:
                p.data = 0.1 * torch.randn(p.shape, generator=g, device=dev).to(torch.bfloat16)
            else:
                t = torch.randn(p.shape, generator=g, device=dev, dtype=torch.bfloat16)
                if p.dim() == 2 and not name.endswith("embed_tokens.weight"):
                    t.mul_(p.shape[1] ** -0.5)
                elif name.endswith("conv1d.weight"):
                    t.mul_(0.5)
                p.data = t
    return m


def _stack_worker(rank, world, port, q):
    """Every rank runs the unsharded stack and its tensor-parallel shard on the same inputs: a
    prefill, then 3 decode steps from one captured CUDA graph (all-reduces inside)."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from visionstack_b200 import Qwen3_5HybridCache
        from visionstack_b200.stack import StackDecodeGraph
        from visionstack_b200.stack_tp import shard_stack
        dev = torch.device("cuda", rank)
        g = torch.Generator(device=dev)
        g.manual_seed(23)
        ids = torch.randint(0, STACK_CFG["vocab_size"], (2, 100), generator=g, device=dev)

        def run(m):
            cache = Qwen3_5HybridCache()
            cache.kv_capacity = 100
            outs = [m(input_ids=ids[:, :96], past_key_values=cache, use_cache=True).last_hidden_state.clone()]
            dg = StackDecodeGraph(m, cache, ids)
            for _ in range(3):
                outs.append(dg.step().clone())
            torch.cuda.synchronize()
            dg.finish()
            return outs, cache

        from visionstack_b200.peer import PeerAllReduce
        peer = PeerAllReduce(max_elems=2 * STACK_CFG["hidden_size"], nblocks=8, device=dev)
        with torch.inference_mode():
            ref, rc = run(_stack_model(dev))
            dist.barrier()
            shd, sc = run(shard_stack(_stack_model(dev), rank, world))
            dist.barrier()
            shp, _ = run(shard_stack(_stack_model(dev), rank, world, peer=peer))
        peer.close()
        errs = [(float((a.float() - b.float()).abs().max()), float((a.float() - b.float()).abs().mean()),
                 float(b.float().abs().max())) for a, b in zip(shd, ref)]
        # decode steps through the peer kernel against the NCCL-sharded stack (both round the sum of the
        # bf16 partials once to bf16; the graph-replayed steps may still order the work differently)
        errs += [(float((a.float() - b.float()).abs().max()), 0.0, 0.0) for a, b in zip(shp[1:], shd[1:])]
        hv = STACK_CFG["linear_num_value_heads"] // world
        s_ref = rc.recurrent_states[0][:, rank * hv:(rank + 1) * hv]
        s_err = float((sc.recurrent_states[0] - s_ref).abs().max() / s_ref.abs().max())
        q.put((rank, errs, s_err))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_tensor_parallel_stack_matches_unsharded():
    """The 4-layer stack cut over 2 GPUs (DeltaNet value heads, attention query heads with their KV
    head, MLP columns, NCCL all-reduce after every mixer and MLP; again with the decode steps' sums
    on the one-shot peer all-reduce) against the unsharded stack: the
    prefill's and three graph-replayed decode steps' final hidden states, and the first DeltaNet
    layer's recurrent state (the same inputs on both sides) as the head slice of the unsharded one.
    bf16 GEMMs cut in N and sums of bf16 partials round differently, so the hidden states are held
    to the stack tests' bf16 bounds (max 0.125, mean 0.01)."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_stack_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, errs, s_err in res:
        for i, (mx, mean, scale) in enumerate(errs[:4]):
            assert mx <= 0.125 and mean <= 0.01, f"rank {rank} step {i}: max {mx}, mean {mean} (|ref| {scale})"
        for i, (mx, _, _) in enumerate(errs[4:]):
            assert mx <= 0.125, f"rank {rank} decode step {i}: peer all-reduce vs NCCL differ by {mx}"
        assert s_err <= 1e-2, f"rank {rank}: first DeltaNet state differs from its head slice by {s_err}"


def _peer_worker(rank, world, port, q):
    """Every rank sums seeded partials with the one-shot peer all-reduce: out of place, in place,
    several sizes, and replayed from a CUDA graph; each result must equal, bit for bit, the fp32
    sum in rank order rounded to bf16 (computed here from every rank's seeded partial)."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from visionstack_b200 import _lib
        from visionstack_b200.peer import PeerAllReduce
        dev = torch.device("cuda", rank)
        peer = PeerAllReduce(max_elems=1 << 17, nblocks=8, device=dev)

        def parts(n, salt):
            return [torch.randn(n, generator=torch.Generator().manual_seed(1000 * salt + 17 * r + n))
                    .to(torch.bfloat16) for r in range(world)]

        def expect(ps):
            acc = torch.zeros(ps[0].shape, dtype=torch.float32)
            for p in ps:
                acc += p.float()
            return acc.to(torch.bfloat16)

        bad = []
        for salt, n in enumerate((8, 8000, 65536, 1 << 17)):
            ps = parts(n, salt)
            x = ps[rank].to(dev)
            out = torch.empty_like(x)
            peer(x, out)
            y = x.clone()
            peer(y)
            torch.cuda.synchronize()
            e = expect(ps)
            if not (torch.equal(out.cpu(), e) and torch.equal(y.cpu(), e)):
                bad.append(f"n={n}")
        # three calls captured in one graph, replayed twice with fresh inputs
        bufs = [torch.empty(4096, dtype=torch.bfloat16, device=dev) for _ in range(3)]
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for b in bufs:
                peer(b)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for b in bufs:
                peer(b)
        for rep in range(2):
            pss = [parts(4096, 10 + 3 * rep + i) for i in range(3)]
            for b, ps in zip(bufs, pss):
                b.copy_(ps[rank].to(dev))
            graph.replay()
            torch.cuda.synchronize()
            for i, (b, ps) in enumerate(zip(bufs, pss)):
                if not torch.equal(b.cpu(), expect(ps)):
                    bad.append(f"graph replay {rep} call {i}")
        del graph
        err = _lib.device_error()
        peer.close()
        q.put((rank, bad, err))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_peer_allreduce_is_exact():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_peer_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, bad, err in res:
        assert not bad and err == 0, f"rank {rank}: {bad}, device error {err:#x}"
