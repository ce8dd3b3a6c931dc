"""Benchmark of the B200 Gated DeltaNet token mixer.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload (one GPU): the single-token decode step of one DeltaNet
layer at batch 64, hidden 2048, 16 key heads / 32 value heads, d_k = d_v = 128,
bf16 activations and an fp32 recurrent state (128 MiB).  Every decode step is
one fused kernel launch that takes the step's projection outputs to the gated
RMSNorm output, updating the recurrent state in place.  One bench step is a
run of 512 such decode steps, captured once as a CUDA graph and replayed; K
bench steps are timed.  ``value`` is decode steps per second, ``ms_per_step``
the time of one bench step (512 launches), ``ms_per_decode_step`` that of one
launch, ``gpu_launches`` K x 512.  Four rotating state slots (4 x 134 MB) keep
every step's state traffic out of the 126 MB L2.

With ``--gpus N`` (torchrun, one rank per GPU) the value heads are sharded:
rank r owns value heads [r*32/N, (r+1)*32/N) and the key heads they read; the
token mixer needs no exchange between ranks (each (batch, head) chain is
independent).  The global batch grows with N (64 N decode rows, 8 N prefill
rows, 16 N rollback rows), so every GPU keeps the single-GPU amount of work
(weak scaling), and ``value`` is the whole job's rate in units of the
single-GPU workload (B64 decode steps per second).

Also reported, as objects of the same line: the chunked-prefill workload
(batch 8 x 8192 tokens), the speculative verify + rollback workload (batch 16,
4-token drafts), the whole head-sharded layer with its NCCL all-reduce at
strong and weak scaling (``sharded_layer``), at one GPU the prefix-cache
snapshot / restore of a 36-layer stack's states (``prefix_snapshot``), and the
48-layer hybrid stack (``stack``, tensor-parallel over the run's GPUs); the roofline of the dominant kernel; an
end-to-end number through the public API with host buffers; the CPU oracle
timed on the host's cores (decode, prefill and the configs[0] layer case);
and SM clocks sampled during the timed region.

``--impl reference`` times the CPU restatement of the reference path (the
numpy oracle) on the host cores, on the same decode workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

from visionstack_b200 import workloads as W  # noqa: E402

FALLBACK_HBM_GBS = 6650.0
DECODE_RUN_STEPS = 512  # the decode workload: 512 single-token steps per bench step
FALLBACK_BF16_TFLOPS = 1590.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-prefill", action="store_true", help="skip the secondary prefill measurement")
    ap.add_argument("--no-decode", action="store_true", help="only the prefill measurement (for profiling)")
    ap.add_argument("--prefill-batch", type=int, default=8)
    ap.add_argument("--prefill-seq", type=int, default=8192)
    ap.add_argument("--no-rollback", action="store_true", help="skip the secondary rollback measurement")
    ap.add_argument("--no-stack", action="store_true",
                    help="skip the secondary 48-layer hybrid stack measurement (B32: prefill 4096, decode 256; "
                         "tensor-parallel over the GPUs of the run)")
    ap.add_argument("--no-sharded", action="store_true",
                    help="skip the head-sharded layer measurement (projections, mixer, out_proj, all-reduce)")
    ap.add_argument("--no-prefix-snapshot", action="store_true",
                    help="skip the prefix-cache snapshot/restore measurement (run at 1 GPU only)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-sample-s", type=float, default=12.0, help="seconds of CPU work for the CPU baseline")
    return ap.parse_args()


# ----------------------------------------------------------------------------
# algorithmic work (per launch)
# ----------------------------------------------------------------------------

def decode_bytes(B: int, hk: int, hv: int, d: int, K: int, act_bytes: int = 2) -> int:
    """Bytes one decode launch must move: state read+write, conv state
    read+write, conv weights, projection outputs in, gated-norm output out."""
    conv_ch = 2 * hk * d + hv * d
    state = 2 * B * hv * d * d * 4
    conv_state = 2 * B * conv_ch * (K - 1) * act_bytes
    conv_w = conv_ch * K * act_bytes
    inputs = B * (conv_ch + hv * d + 2 * hv) * act_bytes
    out = B * hv * d * act_bytes
    return state + conv_state + conv_w + inputs + out


def prefill_flops(B: int, T: int, hv: int, d: int, C: int = 64) -> float:
    """Contraction FLOPs of the chunked form per token and head:
    K K^T and Q K^T (2*2*C*d), T [U | W] (2*C*2d), P v_new (2*C*d), W S, Q S,
    K^T v_new (3*2*d*d)."""
    return float(B) * T * hv * (2 * C * (3 * d + 2 * d) + 6 * d * d)


def prefill_min_bytes(B: int, T: int, hk: int, hv: int, d: int, K: int = 4) -> int:
    conv_ch = 2 * hk * d + hv * d
    per_tok = (conv_ch + hv * d + 2 * hv + hv * d) * 2
    return B * T * per_tok + B * hv * d * d * 4 + B * conv_ch * (K - 1) * 2


def rollback_bytes(B: int, hk: int, hv: int, d: int, T: int, K: int = 4, act_bytes: int = 2) -> int:
    """Bytes one verify + accept step must move: the starting state read once,
    the states after each of the T draft tokens written once (the slots), the
    conv state read and T conv snapshots written, conv weights, projection
    outputs in, gated-norm output out, slot table and accepted counts."""
    conv_ch = 2 * hk * d + hv * d
    state = B * hv * d * d * 4 * (1 + T)
    conv_state = B * conv_ch * (K - 1) * act_bytes * (1 + T)
    conv_w = conv_ch * K * act_bytes
    inputs = B * T * (conv_ch + hv * d + 2 * hv) * act_bytes
    out = B * T * hv * d * act_bytes
    table = B * (T + 1) * 4 * 2 + B * 4
    return state + conv_state + conv_w + inputs + out + table


def measured_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) of the decode kernel at
# B64 x 32 heads, recorded from one ncu capture of this kernel (the capture command and its
# summary are in the profiles folder).  A recorded constant, not measured by this run: ncu
# cannot run inside a timed benchmark.
DECODE_B64_TRAFFIC_RECORDED = 218625024


# ----------------------------------------------------------------------------
# clocks during the timed region (NVML, read only)
# ----------------------------------------------------------------------------

_REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
            0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting", 0x1: "gpu_idle"}


class ClockSampler:
    def __init__(self, device_index: int, period_s: float = 0.005):
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            idx = device_index
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            if vis:
                ids = [v.strip() for v in vis.split(",") if v.strip()]
                if device_index < len(ids) and ids[device_index].isdigit():
                    idx = int(ids[device_index])
            self._h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self._nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nv = None
        self.period = period_s

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                fn = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                    getattr(nv, "nvmlDeviceGetCurrentClocksThrottleReasons")
                r = fn(self._h)
                for bit, name in _REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self._nv is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": float(statistics.median(self.samples)), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons - {"gpu_idle"}), "samples": len(self.samples)}


# ----------------------------------------------------------------------------
# CPU side: oracle timings (CPU baseline and the reference arm)
# ----------------------------------------------------------------------------

def cpu_decode_rate(sample_s: float, threads: int):
    """Time the oracle's decode step (numpy restatement of the reference,
    deltanet.py:165-233 + conv + gated norm) at the full decode batch (B64), the
    rows split into ``threads`` slices run concurrently on host threads (numpy
    releases the GIL inside its array operations; BLAS held to one thread per
    slice).  Returns (steps/s, steps, seconds, threads used)."""
    from concurrent.futures import ThreadPoolExecutor

    from threadpoolctl import threadpool_limits

    from oracle import gdn_oracle as O

    wl = W.WORKLOADS["decode"]
    s = wl.shape
    p = W.make_layer_params(s, wl.w_seed, "bf16")
    rng = np.random.default_rng(wl.x_seed)
    B = wl.batch
    f = lambda *sh, sc=1.0: W.cast(sc * rng.standard_normal(sh).astype(np.float32), "bf16")  # noqa: E731
    mixed, z, a, b = f(B, 1, s.conv_dim, sc=0.7), f(B, 1, s.num_v_heads, s.head_v_dim), f(B, 1, s.num_v_heads), \
        f(B, 1, s.num_v_heads)
    st = W.make_decode_states(wl)
    P = max(1, min(threads, B))
    cut = [B * i // P for i in range(P + 1)]
    conv = [st["conv"][cut[k]:cut[k + 1]].copy() for k in range(P)]
    rec = [st["recurrent"][cut[k]:cut[k + 1]].copy() for k in range(P)]

    def work(k):
        r0, r1 = cut[k], cut[k + 1]
        _, conv[k], rec[k], _, _ = O.mixer_forward(s, mixed[r0:r1], z[r0:r1], a[r0:r1], b[r0:r1], p["conv1d.weight"],
                                                   p["A_log"], p["dt_bias"], p["norm.weight"], "bf16", conv[k],
                                                   rec[k], chunk=False)

    with threadpool_limits(limits=1, user_api="blas"), ThreadPoolExecutor(P) as ex:
        list(ex.map(work, range(P)))  # warm-up
        n, t0 = 0, time.perf_counter()
        while True:
            list(ex.map(work, range(P)))
            n += 1
            el = time.perf_counter() - t0
            if el >= sample_s or n >= 400:
                break
    return n / el, n, el, P


def cpu_prefill_rate(threads: int, rows: int = 8, T: int = 1024):
    """The oracle's chunked prefill (deltanet.py:236-407 + conv + gated norm) on ``rows`` batch rows
    of the prefill workload's layout (16 / 32 heads, d 128, bf16), T tokens each, one row per host
    thread.  The chunked algorithm's cost is linear in the tokens, so tokens/s of this sample is
    the rate at the full batch 8 x 8192.  Returns (tokens/s, seconds, threads used)."""
    from concurrent.futures import ThreadPoolExecutor

    from threadpoolctl import threadpool_limits

    from oracle import gdn_oracle as O

    s = W.SHAPE_QWEN
    p = W.make_layer_params(s, 1, "bf16")
    P = max(1, min(threads, rows))
    rng = np.random.default_rng(3)
    f = lambda *sh, sc=1.0: W.cast(sc * rng.standard_normal(sh).astype(np.float32), "bf16")  # noqa: E731
    ins = [(f(1, T, s.conv_dim, sc=0.7), f(1, T, s.num_v_heads, s.head_v_dim), f(1, T, s.num_v_heads),
            f(1, T, s.num_v_heads)) for _ in range(rows)]

    def work(k):
        mixed, z, a, b = ins[k]
        O.mixer_forward(s, mixed, z, a, b, p["conv1d.weight"], p["A_log"], p["dt_bias"], p["norm.weight"], "bf16")

    blas = max(1, threads // P)
    with threadpool_limits(limits=blas, user_api="blas"), ThreadPoolExecutor(P) as ex:
        t0 = time.perf_counter()
        list(ex.map(work, range(rows)))
        el = time.perf_counter() - t0
    return rows * T / el, el, P * blas


def cpu_layer_cpu_plumbing():
    """The reference's CPU-runnable case: one fp32 layer, batch 1 x 256 tokens, hidden 1024,
    8 / 8 heads of 128, through the oracle's layer forward (projections, conv, chunked delta rule,
    gated norm, out_proj, hybrid-cache side effects), then a 16-token decode continuation.
    Returns (prefill ms, decode ms per token)."""
    from oracle import gdn_oracle as O

    wl = W.WORKLOADS["cpu_plumbing"]
    p = W.make_layer_params(wl.shape, wl.w_seed, "f32")
    x = W.make_hidden(wl)
    cache = O.OracleCache()
    t0 = time.perf_counter()
    O.deltanet_layer_forward(p, wl.shape, x, "f32", cache=cache)
    t_pre = time.perf_counter() - t0
    cache.past_seen_tokens = wl.seq_len
    xs = [W.make_hidden(wl, seq_len=1, seed_offset=i + 1) for i in range(16)]
    t0 = time.perf_counter()
    for xd in xs:
        O.deltanet_layer_forward(p, wl.shape, xd, "f32", cache=cache)
        cache.past_seen_tokens += 1
    t_dec = (time.perf_counter() - t0) / 16
    return t_pre * 1e3, t_dec * 1e3


def cpu_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_baselines(args, full: bool):
    """The CPU restatement of the reference path (the numpy oracle) timed on this host's cores:
    the decode workload (B64), and with ``full`` also the prefill workload's per-token rate and
    the reference's CPU-runnable layer case."""
    threads = cpu_cores()
    rate, n, el, P = cpu_decode_rate(args.cpu_sample_s, threads)
    out = {"value": rate, "unit": "steps/s", "cores": P, "kind": "port",
           "sample": f"{n} decode steps of the numpy oracle at B64 x 32 heads ({el:.1f} s), the 64 rows split "
                     f"over {P} host threads (BLAS one thread each)"}
    if full:
        tps, pel, pc = cpu_prefill_rate(threads)
        out["prefill"] = {"value": tps, "unit": "tokens/s", "cores": pc, "kind": "port",
                          "sample": f"the numpy oracle's chunked prefill on 8 rows x 1024 tokens of the prefill "
                                    f"layout ({pel:.1f} s), one row per host thread; the cost is linear in the "
                                    f"tokens, so this is the rate at 8 x 8192"}
        pre_ms, dec_ms = cpu_layer_cpu_plumbing()
        out["cpu_plumbing_layer"] = {"prefill_ms": pre_ms, "decode_ms_per_token": dec_ms, "cores": 1,
                                     "kind": "port",
                                     "sample": "one fp32 layer, B1 x 256 tokens, hidden 1024, 8 / 8 heads of 128, "
                                               "then 16 decode tokens (numpy, BLAS on the host cores)"}
    return out


def run_reference(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    base = cpu_baselines(args, full=True)
    rate = base["value"]
    line = {
        "metric": "DeltaNet decode steps/s (B64, 16/32 heads, d128, bf16, fp32 state)",
        "value": rate, "unit": "steps/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": DECODE_RUN_STEPS * 1000.0 / rate, "ms_per_decode_step": 1000.0 / rate,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded numpy)", "impl": "reference",
        "config": decode_config(args.gpus),
        "cpu_baseline": base,
        "e2e": {"value": rate, "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def decode_config(n: int):
    return {"workload": "decode: B64 per GPU, hidden 2048, 16 k-heads / 32 v-heads, d128, conv 4; one bench step "
                        f"= {DECODE_RUN_STEPS} single-token steps (one kernel launch each), states updated in place",
            "global_batch": 64 * n, "seq_len": 1,
            "parallelism": f"value-head sharding x{n}, batch {64 * n} (64 per GPU)" if n > 1 else "single GPU",
            "l2": "inputs larger than L2: 4 rotating 134 MB state slots"}


# ----------------------------------------------------------------------------
# GPU side
# ----------------------------------------------------------------------------

def build_shard_layer(torch, rank: int, world: int, dev):
    """Layer holding the value-head shard of rank ``rank``: its conv channels
    (q/k of its key heads, v of its value heads), A_log, dt_bias, norm."""
    from visionstack_b200 import Qwen3_5GatedDeltaNet, Qwen3_5TextConfig
    from visionstack_b200.sharding import shard_params
    s = W.SHAPE_QWEN
    full = W.make_layer_params(s, 1, "bf16")
    params, local = shard_params(full, s, rank, world)
    cfg = Qwen3_5TextConfig(hidden_size=s.hidden_size, linear_num_key_heads=local.num_k_heads,
                            linear_num_value_heads=local.num_v_heads, linear_key_head_dim=s.head_k_dim,
                            linear_value_head_dim=s.head_v_dim)
    m = Qwen3_5GatedDeltaNet(cfg, 0)
    with torch.no_grad():
        for name, p in m.named_parameters():
            t = torch.from_numpy(params[name])
            p.data = t if name in ("A_log", "dt_bias") else t.to(torch.bfloat16)
    return m.to(dev), local


def run_ours(args, rank: int, world: int) -> None:
    import torch
    import torch.distributed as dist

    from visionstack_b200 import _lib

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    lib = _lib.load()
    m, local = build_shard_layer(torch, rank, world, dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    if args.no_decode:
        pf = run_prefill(torch, dist, m, local, dev, world, barrier, args.prefill_batch * world, args.prefill_seq)
        if rank == 0:
            print(json.dumps({"prefill": pf}), flush=True)
        return
    B = 64 * world  # global batch: every rank has all rows for its value heads
    hv, hk, d = local.num_v_heads, local.num_k_heads, local.head_k_dim
    conv_dim, vdim = local.conv_dim, local.value_dim
    NSLOT, NIN = 4, 64
    g = torch.Generator(device=dev)
    g.manual_seed(2 + 1009 * rank)
    with torch.no_grad():
        x = torch.randn(NIN * B, W.SHAPE_QWEN.hidden_size, generator=g, device=dev).to(torch.bfloat16)
        mixed = (x @ m.in_proj_qkv.weight.t()).view(NIN, B, 1, conv_dim)
        z = (x @ m.in_proj_z.weight.t()).view(NIN, B, 1, vdim)
        bb = (x @ m.in_proj_b.weight.t()).view(NIN, B, 1, hv)
        aa = (x @ m.in_proj_a.weight.t()).view(NIN, B, 1, hv)
        del x
        states = [0.02 * torch.randn(B, hv, d, d, generator=g, device=dev) for _ in range(NSLOT)]
        convs = [[torch.randn(B, conv_dim, 3, generator=g, device=dev).to(torch.bfloat16) for _ in range(2)]
                 for _ in range(NSLOT)]
        out = torch.empty(B, 1, vdim, dtype=torch.bfloat16, device=dev)

    def step(i):
        slot, j = i % NSLOT, i % NIN
        cin, cout = convs[slot][(i // NSLOT) % 2], convs[slot][(i // NSLOT + 1) % 2]
        m.mixer(mixed[j], z[j], bb[j], aa[j], conv_state=cin, rec_state=states[slot], conv_state_out=cout,
                rec_state_out=states[slot], out=out, token_by_token=True)

    # One bench step = the decode workload's run of RUN single-token steps (RUN kernel launches,
    # captured once into a CUDA graph); W untimed replays, then K timed ones.
    K, Wm = args.steps, max(3, args.warmup)
    RUN = DECODE_RUN_STEPS
    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        for i in range(4):
            step(i)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(RUN):
            step(i)
    torch.cuda.synchronize(dev)
    for _ in range(Wm):
        graph.replay()
    torch.cuda.synchronize(dev)

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(dev.index)
    barrier()
    with sampler:
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for _ in range(K):
                graph.replay()
            ev1.record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    ms_total = ev0.elapsed_time(ev1)
    t_local = torch.tensor([ms_total], device=dev)
    if world > 1:
        dist.all_reduce(t_local, op=dist.ReduceOp.MAX)
    ms_total = float(t_local.item())
    ms_run = ms_total / K            # one bench step: RUN decode launches
    ms_step = ms_run / RUN           # one decode step
    del graph

    # end to end through the public API: every step copies its projection
    # outputs (packed [mixed | z | b | a] rows, one copy) from pinned host memory,
    # calls the mixer, and copies the gated-norm output back to pinned host
    # memory.  Copies run on two copy streams over NB device buffers, so step i's
    # input copy starts once step i - NB's kernel is done with its buffer: with eight
    # buffers every copy a step's kernel waits for finished a step earlier, and the
    # kernels follow one another as in the device-timed loop.
    K_e2e = min(K, 1000)
    wdt = conv_dim + vdim + 2 * hv
    with torch.no_grad():
        packed = torch.cat([mixed[:, :, 0], z[:, :, 0], bb[:, :, 0], aa[:, :, 0]], dim=-1)  # [NIN, B, wdt]
    h_in = packed.cpu().pin_memory()
    NB = 8
    d_in = [torch.empty(B, 1, wdt, dtype=torch.bfloat16, device=dev) for _ in range(NB)]
    d_out = [torch.empty(B, 1, vdim, dtype=torch.bfloat16, device=dev) for _ in range(NB)]
    h_out = [torch.empty(B, 1, vdim, dtype=torch.bfloat16).pin_memory() for _ in range(NB)]
    s_h2d, s_d2h = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev_ready = [torch.cuda.Event() for _ in range(NB)]
    ev_used = [torch.cuda.Event() for _ in range(NB)]
    ev_back = [torch.cuda.Event() for _ in range(NB)]
    h2d = wdt * B * 2
    d2h = B * vdim * 2

    def bind(x):
        xm, xz = x[..., :conv_dim], x[..., conv_dim:conv_dim + vdim]
        xb, xa = x[..., conv_dim + vdim:conv_dim + vdim + hv], x[..., conv_dim + vdim + hv:]
        return lambda cin, st, cout, o: plan(xm, xz, xb, xa, cin, st, cout, st, o, stream_handle)

    stream_handle = stream.cuda_stream
    plan = None
    views = None

    def e2e_run(n, first):
        # the side streams join whatever stream the steps are issued from (a graph capture included)
        ev_fork = torch.cuda.Event()
        ev_fork.record(stream)
        s_h2d.wait_event(ev_fork)
        s_d2h.wait_event(ev_fork)
        for i in range(n):
            jb, slot = i % NB, (first + i) % NSLOT
            with torch.cuda.stream(s_h2d):
                if i >= NB:
                    s_h2d.wait_event(ev_used[jb])
                d_in[jb][:, 0].copy_(h_in[(first + i) % NIN], non_blocking=True)
                ev_ready[jb].record(s_h2d)
            stream.wait_event(ev_ready[jb])
            if i >= NB:
                stream.wait_event(ev_back[jb])
            x = d_in[jb]
            cin = convs[slot][((first + i) // NSLOT) % 2]
            cout = convs[slot][((first + i) // NSLOT + 1) % 2]
            with torch.cuda.stream(stream):
                views[jb](cin, states[slot], cout, d_out[jb])
                ev_used[jb].record(stream)
            with torch.cuda.stream(s_d2h):
                s_d2h.wait_event(ev_used[jb])
                h_out[jb].copy_(d_out[jb], non_blocking=True)
                ev_back[jb].record(s_d2h)
        for j in range(max(0, n - NB), n):  # every output copy of the run has landed
            stream.wait_event(ev_back[j % NB])

    plan = m.mixer_plan(B, 1, torch.bfloat16, dev, token_by_token=True)
    views = [bind(x) for x in d_in]
    e2e_run(4, 0)
    torch.cuda.synchronize(dev)
    # Serving-style decode loop: GE steps captured into one CUDA graph (each step still copies
    # its own inputs from pinned host memory, calls the plan, and copies its output back), the
    # graph replayed to cover the timed steps; this takes the host's per-step issue cost out.
    GE = 64  # a multiple of 2 x NSLOT and of NB: every replay leaves the conv-state ping-pong and the
    # buffer rotation where they began
    g_e2e = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_e2e, stream=stream):
        e2e_run(GE, 4)
    g_e2e.replay()
    torch.cuda.synchronize(dev)
    n_rep = max(1, K_e2e // GE)
    K_e2e = n_rep * GE
    barrier()
    with torch.cuda.stream(stream):
        ev0.record(stream)
        for _ in range(n_rep):
            g_e2e.replay()
        ev1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    del g_e2e
    t_e2e = torch.tensor([ev0.elapsed_time(ev1) / K_e2e], device=dev)
    if world > 1:
        dist.all_reduce(t_e2e, op=dist.ReduceOp.MAX)
    e2e_ms = float(t_e2e.item())

    # secondary: chunked prefill (batch 8 x 8192 tokens, all heads of the shard)
    prefill = None
    if not args.no_prefill:
        prefill = run_prefill(torch, dist, m, local, dev, world, barrier, args.prefill_batch * world,
                              args.prefill_seq)

    # secondary: speculative verify + rollback on per-row state slots
    rollback = None
    if not args.no_rollback:
        rollback = run_rollback(torch, dist, m, local, dev, world, barrier)

    sharded = None
    if not args.no_sharded:
        sharded = run_sharded_layer(torch, dist, m, local, rank, world, dev, barrier)

    prefix_snap = None
    if not args.no_prefix_snapshot and world == 1:
        prefix_snap = run_prefix_snapshot(torch, m, local, dev)

    stack = None
    if not args.no_stack:
        if world == 1:
            try:
                stack = run_stack(torch, dist, dev, rank, world, barrier)
            except Exception as e:  # the stack is a secondary measurement: never lose the line to it
                stack = {"error": f"{type(e).__name__}: {e}"[:300]}
        else:  # every rank takes the same collective steps; an error ends the job
            stack = run_stack(torch, dist, dev, rank, world, barrier)

    if rank != 0:
        return
    hbm, tflops, src = measured_peaks()
    bytes_launch = decode_bytes(B, hk, hv, d, 4)
    achieved = bytes_launch / (ms_step * 1e-3) / 1e9
    traffic = DECODE_B64_TRAFFIC_RECORDED if world == 1 else None
    line = {
        "metric": "DeltaNet decode steps/s (B64, 16/32 heads, d128, bf16, fp32 state)",
        "value": world * 1000.0 / ms_step, "unit": "steps/s", "n_gpus": world, "steps": K, "warmup": Wm,
        "ms_per_step": ms_run, "ms_per_decode_step": ms_step, "decode_steps_per_bench_step": RUN,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded torch.randn on device)", "config": decode_config(world),
        "gpu_launches": K * RUN,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "traffic": traffic,
                     "traffic_source": "recorded constant from one ncu capture of this kernel at B64 (not "
                                       "measured by this run)" if traffic else None,
                     "peak_source": src, "bytes_per_launch": bytes_launch,
                     "kernel": "gdn::dtma::decode_tma_kernel<128,1,bf16> (2 groups x 256 threads, 1 CTA/SM)"},
        "e2e": {"value": world * 1000.0 / e2e_ms, "unit": "steps/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "path": "Qwen3_5GatedDeltaNet.mixer_plan -> gdn_mixer_decode in CUDA graphs of 64 steps; every "
                        "step: H2D of its packed inputs from pinned host memory, the plan call, D2H of its "
                        "output; copies on two copy streams over 8 device buffers"},
        "clocks": sampler.summary(),
    }
    if prefill is not None:
        line["prefill"] = prefill
    if rollback is not None:
        line["rollback"] = rollback
    if sharded is not None:
        line["sharded_layer"] = sharded
    if prefix_snap is not None:
        line["prefix_snapshot"] = prefix_snap
    if stack is not None:
        line["stack"] = stack
    if world == 1 and not args.no_cpu_baseline:
        base = cpu_baselines(args, full=prefill is not None)
        if prefill is not None and "prefill" in base:
            prefill["cpu_baseline"] = base.pop("prefill")
        line["cpu_baseline"] = base
    print(json.dumps(line), flush=True)


def run_prefix_snapshot(torch, m, local, dev, layers=36, prefix=4096, checkpoints=(1024, 2048, 3072)):
    """Prefix-cache snapshot and splice of the DeltaNet states of a 36-layer stack at B1 (current
    states at 4096 tokens + checkpoints at 1024/2048/3072: 4 x 36 x (2 MiB recurrent + 48 KiB conv)),
    seeded random states.  The snapshot's device-to-host copies run on the copy stream into one
    pinned arena; the restore copies host-to-device on the same stream.  Also timed: 64 B64 decode
    steps (one CUDA graph) alone and with a snapshot in flight beside them."""
    from visionstack_b200 import Qwen3_5HybridCache, snapshot_prefix_state
    from visionstack_b200.prefix import copy_stream
    hv, d = local.num_v_heads, local.head_k_dim
    g = torch.Generator(device=dev)
    g.manual_seed(9)
    cache = Qwen3_5HybridCache()
    for l in range(layers):
        cache.conv_states[l] = torch.randn(1, local.conv_dim, 3, generator=g, device=dev).to(torch.bfloat16)
        cache.recurrent_states[l] = 0.02 * torch.randn(1, hv, d, d, generator=g, device=dev)
        for cp in checkpoints:
            cache.conv_checkpoints.setdefault(cp, {})[l] = cache.conv_states[l].clone()
            cache.recurrent_checkpoints.setdefault(cp, {})[l] = cache.recurrent_states[l].clone()
    toks = list(range(prefix))
    cs = copy_stream(dev)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]

    def snap_once():
        torch.cuda.synchronize(dev)
        ev[0].record(cs)
        st = snapshot_prefix_state(toks, None, cache)
        ev[1].record(cs)
        st.synchronize()
        return st, ev[0].elapsed_time(ev[1])

    for _ in range(2):
        st, _ = snap_once()
    st, d2h_ms = min((snap_once() for _ in range(3)), key=lambda r: r[1])
    nbytes = sum(t.numel() * t.element_size() for mp in st.recurrent_checkpoints.values() for t in mp.values()) + \
        sum(t.numel() * t.element_size() for mp in st.conv_checkpoints.values() for t in mp.values())
    # restore at 3072: every layer's checkpoint states back on the device
    h2d = []
    for _ in range(4):
        torch.cuda.synchronize(dev)
        ev[2].record(cs)
        rc, _, off = st.restore(dev, snap_len=3072)
        ev[3].record(cs)
        torch.cuda.synchronize(dev)
        h2d.append(ev[2].elapsed_time(ev[3]))
    restore_ms = min(h2d[1:])
    rbytes = sum(t.numel() * t.element_size() for t in list(rc.recurrent_states.values()) +
                 list(rc.conv_states.values()))
    ok = all(torch.equal(rc.recurrent_states[l].cpu(), st.recurrent_checkpoints[3072][l]) for l in (0, layers - 1))

    # overlap: 64 decode steps at B64 alone, then with a snapshot of the same states in flight
    Bd = 64
    with torch.no_grad():
        x = torch.randn(Bd, 1, W.SHAPE_QWEN.hidden_size, generator=g, device=dev).to(torch.bfloat16)
        mixed, z, bb, aa = m.project(x)
    S = 0.02 * torch.randn(Bd, hv, d, d, generator=g, device=dev)
    cv = [torch.zeros(Bd, local.conv_dim, 3, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        for i in range(3):
            m.mixer(mixed, z, bb, aa, conv_state=cv[i % 2], rec_state=S, conv_state_out=cv[(i + 1) % 2],
                    rec_state_out=S, token_by_token=True)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(64):
            m.mixer(mixed, z, bb, aa, conv_state=cv[i % 2], rec_state=S, conv_state_out=cv[(i + 1) % 2],
                    rec_state_out=S, token_by_token=True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def decode_ms(with_snapshot):
        torch.cuda.synchronize(dev)
        with torch.cuda.stream(stream):
            if with_snapshot:
                snap = snapshot_prefix_state(toks, None, cache)
            e0.record(stream)
            graph.replay()
            e1.record(stream)
        torch.cuda.synchronize(dev)
        if with_snapshot:
            snap.synchronize()
        return e0.elapsed_time(e1)

    decode_ms(False)
    alone = min(decode_ms(False) for _ in range(3))
    beside = min(decode_ms(True) for _ in range(3))
    del graph
    return {"workload": f"prefix snapshot of {layers} DeltaNet layers at B1: current states at {prefix} tokens + "
                        f"checkpoints at {list(checkpoints)} (2 MiB recurrent + 48 KiB conv per layer and offset); "
                        f"restore at 3072",
            "snapshot_bytes": nbytes, "d2h_ms": d2h_ms, "d2h_gbs": nbytes / (d2h_ms * 1e-3) / 1e9,
            "restore_bytes": rbytes, "h2d_ms": restore_ms, "h2d_gbs": rbytes / (restore_ms * 1e-3) / 1e9,
            "restore_bit_exact": bool(ok),
            "decode_64_steps_ms": {"alone": alone, "with_snapshot_in_flight": beside, "ratio": beside / alone},
            "path": "visionstack_b200.prefix.snapshot_prefix_state / PinnedPrefixState.restore: copies on a "
                    "dedicated copy stream, one pinned arena per snapshot, no host synchronisation"}


def run_prefill(torch, dist, m, local, dev, world, barrier, B=8, T=8192):
    hv, hk, d = local.num_v_heads, local.num_k_heads, local.head_k_dim
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    with torch.no_grad():
        x = torch.randn(B, T, W.SHAPE_QWEN.hidden_size, generator=g, device=dev).to(torch.bfloat16)
        mixed, z, bb, aa = m.project(x)
        del x
    out = torch.empty(B, T, local.value_dim, dtype=torch.bfloat16, device=dev)
    S = torch.empty(B, hv, d, d, device=dev)
    cs = torch.empty(B, local.conv_dim, 3, dtype=torch.bfloat16, device=dev)

    def once():
        m.mixer(mixed, z, bb, aa, conv_state_out=cs, rec_state_out=S, out=out, token_by_token=False)

    for _ in range(3):
        once()
    reps = 5
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    ev0.record()
    for _ in range(reps):
        once()
    ev1.record()
    torch.cuda.synchronize(dev)
    barrier()
    t = torch.tensor([ev0.elapsed_time(ev1) / reps], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    _, tflops, src = measured_peaks()
    fl = prefill_flops(B, T, hv, d)
    ach = fl / (ms * 1e-3) / 1e12
    return {"workload": f"chunked prefill: B{B} x T{T}, 16 k-heads / 32 v-heads (sharded), d128, bf16",
            "tokens_per_s": B * T / (ms * 1e-3), "ms_per_launch": ms,
            "roofline": {"bound": "tensor", "achieved": ach, "peak": tflops, "unit": "TFLOP/s",
                         "frac": ach / tflops, "peak_source": src, "flops_per_launch": fl,
                         "min_bytes_per_launch": prefill_min_bytes(B, T, hk, hv, d),
                         "kernel": "gdn::pseq::prefill_seq_kernel (tcgen05 bf16 hi+lo and tf32, state in tensor memory, 1 CTA per (batch, head)) after gdn::pprep::prefill_prep_kernel"}}


def run_stack(torch, dist, dev, rank, world, barrier):
    """The 48-layer hybrid stack (36 Gated DeltaNet layers on the CUDA token mixer, 12 gated
    attention layers and all MLPs on library kernels), random bf16 weights, B32: a 4096-token
    prefill into a hybrid cache, then 256 decode steps of random token ids.  The prefill is eager
    PyTorch around the mixer; the decode steps replay one captured CUDA graph (static KV buffers,
    the position on the device); the decode time is that of the replayed steps.  With N ranks the
    stack is tensor-parallel (``stack_tp.shard_stack``: DeltaNet value heads, attention query
    heads with the KV heads they read, MLP columns; two NCCL all-reduces per layer, inside the
    decode graph too) at the same batch (strong scaling); times are the max over ranks."""
    from visionstack_b200 import Qwen3_5HybridCache, Qwen3_5TextConfig
    from visionstack_b200.stack import Qwen3_5TextModel, StackDecodeGraph
    from visionstack_b200.stack_tp import shard_stack
    cfg = Qwen3_5TextConfig(**W.STACK_48)
    R = W.STACK_48_RUN
    B, P, D = R["batch"], R["prefill"], R["decode"]
    with torch.device("meta"):
        model = Qwen3_5TextModel(cfg)
    model = model.to_empty(device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(R["seed"])
    bf = torch.bfloat16
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith("A_log"):
                p.data = torch.empty(p.shape, device=dev).uniform_(-1.0, 1.0, generator=g)
            elif name.endswith("dt_bias"):
                p.data = torch.zeros(p.shape, device=dev)
            elif name.endswith("linear_attn.norm.weight"):
                p.data = torch.ones(p.shape, device=dev, dtype=bf)
            elif name.endswith("norm.weight") or name.endswith("layernorm.weight"):
                p.data = torch.zeros(p.shape, device=dev, dtype=bf)
            else:
                t = torch.randn(p.shape, generator=g, device=dev, dtype=bf)
                if p.dim() == 2 and not name.endswith("embed_tokens.weight"):
                    t.mul_(p.shape[1] ** -0.5)
                elif name.endswith("conv1d.weight"):
                    t.mul_(0.5)
                p.data = t
    ids = torch.randint(0, cfg.vocab_size, (B, P + D), generator=g, device=dev)
    peer = None
    if world > 1:
        from visionstack_b200.peer import PeerAllReduce
        peer = PeerAllReduce(max_elems=B * cfg.hidden_size, nblocks=32, device=dev)  # the decode steps' sums
        shard_stack(model, rank, world, peer=peer)
        torch.cuda.empty_cache()

    def run(n_pre, n_dec):
        cache = Qwen3_5HybridCache()
        cache.kv_capacity = n_pre + n_dec
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        torch.cuda.synchronize(dev)
        barrier()
        ev[0].record()
        model(input_ids=ids[:, :n_pre], past_key_values=cache, use_cache=True)
        ev[1].record()
        torch.cuda.synchronize(dev)
        # decode: the first step eager (and the graph's capture), the rest replayed from the graph
        dg = StackDecodeGraph(model, cache, ids)
        dg.step()
        torch.cuda.synchronize(dev)
        barrier()
        ev[2].record()
        for _ in range(n_dec - 1):
            dg.step()
        ev[3].record()
        torch.cuda.synchronize(dev)
        dg.finish()
        del dg
        t = _max_over_ranks(torch, dist, world, dev, ev[0].elapsed_time(ev[1]),
                            ev[2].elapsed_time(ev[3]) / (n_dec - 1) * n_dec)
        return t[0], t[1]

    with torch.inference_mode():
        run(256, 4)
        run(P, 8)
        t_pre, t_dec = run(P, D)
    peak_mem = torch.cuda.max_memory_allocated(dev)
    nl = sum(1 for t in cfg.layer_types if t == "linear_attention")
    na = cfg.num_hidden_layers - nl
    # per rank: its weight shard (embedding excluded: one row per token is read), its DeltaNet
    # heads' states, its KV heads' cache; FLOPs of the whole job over the GPUs (each does 1/N)
    params = sum(p.numel() for n, p in model.named_parameters() if not n.endswith("embed_tokens.weight"))
    wbytes = sum(p.numel() * p.element_size() for n, p in model.named_parameters()
                 if not n.endswith("embed_tokens.weight"))
    hv, dk = cfg.linear_num_value_heads // world, cfg.linear_key_head_dim
    conv_dim = (2 * cfg.linear_num_key_heads * dk + cfg.linear_num_value_heads * cfg.linear_value_head_dim) // world
    state_rw = nl * (2 * B * hv * dk * dk * 4 + 2 * B * conv_dim * 3 * 2)
    kv_heads = max(1, cfg.num_key_value_heads // world)
    kv_read = na * B * 2 * (P + D // 2) * kv_heads * cfg.head_dim * 2
    dec_bytes = wbytes + state_rw + kv_read
    ms_dec = t_dec / D
    hbm, tflops, src = measured_peaks()
    attn_fl = na * B * (cfg.num_attention_heads // world) * (P * P / 2) * cfg.head_dim * 4
    pre_fl = 2.0 * params * B * P + attn_fl + nl * prefill_flops(B, P, hv, dk)  # per rank
    del model
    if peer is not None:
        peer.close()
    torch.cuda.empty_cache()
    return {"workload": f"48-layer hybrid stack (36 Gated DeltaNet + 12 gated attention, hidden 2048, MLP 12288, "
                        f"vocab 151936), random bf16 weights, B{B}: prefill {P} tokens then {D} decode steps",
            "world": world,
            "parallelism": "single GPU" if world == 1 else
            f"tensor-parallel over {world} GPUs (DeltaNet value heads, attention query heads with their KV "
            f"heads, MLP columns; an all-reduce after every mixer and MLP: the one-shot NVLink peer kernel "
            f"for the decode steps, NCCL for the prefill), global batch fixed (strong)",
            "prefill_tokens_per_s": B * P / (t_pre * 1e-3), "prefill_ms": t_pre,
            "decode_steps_per_s": 1000.0 / ms_dec, "decode_tokens_per_s": B * 1000.0 / ms_dec,
            "decode_ms_per_step": ms_dec, "peak_memory_gb": peak_mem / 1e9,
            "prefill_roofline": {"bound": "tensor", "achieved": pre_fl / (t_pre * 1e-3) / 1e12, "peak": tflops,
                                 "unit": "TFLOP/s", "frac": pre_fl / (t_pre * 1e-3) / 1e12 / tflops,
                                 "flops_per_gpu": pre_fl, "peak_source": src},
            "decode_roofline": {"bound": "hbm", "achieved": dec_bytes / (ms_dec * 1e-3) / 1e9, "peak": hbm,
                                "unit": "GB/s", "frac": dec_bytes / (ms_dec * 1e-3) / 1e9 / hbm,
                                "bytes_per_step_per_gpu": dec_bytes, "peak_source": src},
            "path": "visionstack_b200.stack.Qwen3_5TextModel (prefill eager, decode from one CUDA graph; with N "
                    "GPUs cut by visionstack_b200.stack_tp.shard_stack); "
                    "DeltaNet layers on gdn_mixer_prefill_ws / gdn_mixer_decode, decode attention on "
                    "gdn_attn_decode, prefill attention on torch SDPA, GEMMs on cuBLAS"}



# ----------------------------------------------------------------------------
# the head-sharded layer: input projections, token mixer, out_proj, all-reduce
# ----------------------------------------------------------------------------

def _allreduce_busbw(nbytes: int, ms: float, world: int) -> float:
    """NCCL-convention bus bandwidth of an all-reduce: bytes * 2 (N - 1) / N / time."""
    return nbytes * 2.0 * (world - 1) / world / (ms * 1e-3) / 1e9 if world > 1 and ms > 0 else 0.0


def _ev_time(torch, fn, reps: int, stream=None) -> float:
    """Mean ms of ``fn`` over ``reps`` calls, CUDA events on the current stream."""
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def _max_over_ranks(torch, dist, world, dev, *vals):
    t = torch.tensor(list(vals), device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.tolist()]


def sharded_decode(torch, dist, m, local, dev, world, barrier, Bg: int, steps: int = 256, graph_steps: int = 32,
                   peer=None):
    """One decode step of the value-head-sharded layer at global batch Bg: this rank's fused input
    projection, the token mixer on its heads (state in place), its out_proj column slice, and the
    all-reduce (bf16 sum) of the [Bg, 1, hidden] partial outputs: NCCL, or with ``peer`` the
    one-shot NVLink kernel (gdn_peer_allreduce_bf16).  Steps replay from CUDA graphs of
    ``graph_steps`` steps; state slots rotate so the states never sit in L2."""
    from visionstack_b200.peer import sum_partials
    hv, d, H = local.num_v_heads, local.head_k_dim, W.SHAPE_QWEN.hidden_size
    state_bytes = Bg * hv * d * d * 4
    nslot = max(2, -(-300_000_000 // state_bytes))
    nslot += nslot % 2
    NIN = 16
    g = torch.Generator(device=dev)
    g.manual_seed(2)
    with torch.no_grad():
        xs = torch.randn(NIN, Bg, 1, H, generator=g, device=dev).to(torch.bfloat16)
        states = [0.02 * torch.randn(Bg, hv, d, d, generator=g, device=dev) for _ in range(nslot)]
        convs = [[torch.zeros(Bg, local.conv_dim, 3, dtype=torch.bfloat16, device=dev) for _ in range(2)]
                 for _ in range(nslot)]
        core = torch.empty(Bg, 1, local.value_dim, dtype=torch.bfloat16, device=dev)
        y = torch.empty(Bg, 1, H, dtype=torch.bfloat16, device=dev)
    w_out = m.out_proj.weight
    plan = m.mixer_plan(Bg, 1, torch.bfloat16, dev, token_by_token=True)

    def step(i, reduce=True):
        slot = i % nslot
        mixed, z, bb, aa = m.project(xs[i % NIN])
        plan(mixed, z, bb, aa, convs[slot][(i // nslot) % 2], states[slot], convs[slot][(i // nslot + 1) % 2],
             states[slot], core)
        torch.matmul(core, w_out.t(), out=y)
        if reduce and world > 1:
            sum_partials(y, peer)

    stream = torch.cuda.Stream(device=dev)
    with torch.no_grad(), torch.cuda.stream(stream):
        for i in range(4):
            step(i)
    torch.cuda.synchronize(dev)
    graphs = {}
    try:
        for reduce in (True, False):
            gr = torch.cuda.CUDAGraph()
            with torch.no_grad(), torch.cuda.graph(gr, stream=stream):
                for i in range(graph_steps):
                    step(i, reduce)
            graphs[reduce] = gr
        mode = "CUDA graphs"
    except Exception as e:  # a capture the library refuses: time the eager loop instead
        graphs = {}
        mode = f"eager ({type(e).__name__})"
    torch.cuda.synchronize(dev)
    reps = max(1, steps // graph_steps)

    def run(reduce):
        if graphs:
            graphs[reduce].replay()
        else:
            with torch.no_grad():
                for i in range(graph_steps):
                    step(i, reduce)

    with torch.cuda.stream(stream):
        run(True)
        run(False)
        barrier()
        ms_full = _ev_time(torch, lambda: run(True), reps) / graph_steps
        barrier()
        ms_local = _ev_time(torch, lambda: run(False), reps) / graph_steps
        barrier()
        # the all-reduce of one step's partial outputs, alone: 32 calls replayed from one CUDA graph
        # (as inside the step; an eager loop would time the host's launch path)
        ms_ar = 0.0
        if world > 1:
            gar = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gar, stream=stream):
                for _ in range(32):
                    sum_partials(y, peer)
            gar.replay()
            barrier()
            ms_ar = _ev_time(torch, gar.replay, 8) / 32
            del gar
        barrier()
    graphs.clear()
    ms_full, ms_local, ms_ar = _max_over_ranks(torch, dist, world, dev, ms_full, ms_local, ms_ar)
    ar_bytes = Bg * H * 2
    w_bytes = sum(p.numel() * p.element_size() for n, p in m.named_parameters())
    hbm_bytes = w_bytes + decode_bytes(Bg, local.num_k_heads, hv, d, 4) + 2 * Bg * H * 2
    hbm, _, src = measured_peaks()
    return {"global_batch": Bg, "ms_per_step": ms_full, "steps_per_s": 1000.0 / ms_full,
            "ms_per_step_without_allreduce": ms_local, "allreduce_ms_alone": ms_ar,
            "allreduce_bytes": ar_bytes, "allreduce_busbw_gbs": _allreduce_busbw(ar_bytes, ms_ar, world),
            "roofline": {"bound": "hbm", "bytes_per_gpu_per_step": hbm_bytes,
                         "achieved": hbm_bytes / (ms_full * 1e-3) / 1e9, "peak": hbm, "unit": "GB/s",
                         "frac": hbm_bytes / (ms_full * 1e-3) / 1e9 / hbm, "peak_source": src},
            "allreduce": "one-shot over NVLink peer memory (gdn_peer_allreduce_bf16)" if peer is not None and
            world > 1 else ("NCCL" if world > 1 else None),
            "timing": mode}


def sharded_prefill(torch, dist, m, local, dev, world, barrier, Bg: int, T: int, slabs: int = 4, reps: int = 3):
    """Prefill of the value-head-sharded layer at global batch Bg x T tokens, the sequence cut into
    ``slabs`` T-slabs: per slab this rank's input projection, the token mixer on its heads (states
    handed from slab to slab), its out_proj partial, and that slab's all-reduce issued
    asynchronously, so NCCL's stream reduces slab i while slab i + 1 computes."""
    H = W.SHAPE_QWEN.hidden_size
    hv, d = local.num_v_heads, local.head_k_dim
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    with torch.no_grad():
        x = torch.randn(Bg, T, H, generator=g, device=dev).to(torch.bfloat16)
        S = torch.empty(Bg, hv, d, d, device=dev)
        cs = [torch.empty(Bg, local.conv_dim, 3, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    bounds = [T * i // slabs for i in range(slabs + 1)]
    with torch.no_grad():
        # per slab: a contiguous gated-norm output and a contiguous partial output (NCCL reduces
        # whole tensors; the slabs' reductions stay in flight while the next slab computes)
        core = torch.empty(Bg, bounds[1], local.value_dim, dtype=torch.bfloat16, device=dev)
        ys = [torch.empty(Bg, bounds[i + 1] - bounds[i], H, dtype=torch.bfloat16, device=dev) for i in range(slabs)]
    w_out = m.out_proj.weight

    def once(reduce=True):
        works = []
        with torch.no_grad():
            for i in range(slabs):
                t0, t1 = bounds[i], bounds[i + 1]
                mixed, z, bb, aa = m.project(x[:, t0:t1])
                c = core.view(-1)[:Bg * (t1 - t0) * local.value_dim].view(Bg, t1 - t0, local.value_dim)
                m.mixer(mixed, z, bb, aa, conv_state=cs[(i + 1) % 2] if i else None, rec_state=S if i else None,
                        conv_state_out=cs[i % 2], rec_state_out=S, out=c, token_by_token=False)
                torch.matmul(c, w_out.t(), out=ys[i])
                if reduce and world > 1:
                    works.append(dist.all_reduce(ys[i], op=dist.ReduceOp.SUM, async_op=True))
        for w in works:
            w.wait()

    once()
    once(False)
    torch.cuda.synchronize(dev)
    barrier()
    ms_full = _ev_time(torch, once, reps)
    barrier()
    ms_local = _ev_time(torch, lambda: once(False), reps)
    barrier()
    ms_ar = _ev_time(torch, lambda: [dist.all_reduce(t, op=dist.ReduceOp.SUM) for t in ys], reps) \
        if world > 1 else 0.0
    barrier()
    ms_full, ms_local, ms_ar = _max_over_ranks(torch, dist, world, dev, ms_full, ms_local, ms_ar)
    _, tflops, src = measured_peaks()
    gemm_fl = 2.0 * Bg * T * H * (local.conv_dim + local.value_dim + 2 * hv) + 2.0 * Bg * T * local.value_dim * H
    fl = gemm_fl + prefill_flops(Bg, T, hv, d)
    ar_bytes = Bg * T * H * 2
    return {"global_batch": Bg, "seq_len": T, "slabs": slabs, "ms_per_call": ms_full,
            "tokens_per_s": Bg * T / (ms_full * 1e-3), "ms_per_call_without_allreduce": ms_local,
            "allreduce_ms_alone": ms_ar, "allreduce_bytes": ar_bytes,
            "allreduce_busbw_gbs": _allreduce_busbw(ar_bytes, ms_ar, world),
            "allreduce_exposed_ms": max(0.0, ms_full - ms_local),
            "roofline": {"bound": "tensor", "flops_per_gpu": fl, "achieved": fl / (ms_full * 1e-3) / 1e12,
                         "peak": tflops, "unit": "TFLOP/s", "frac": fl / (ms_full * 1e-3) / 1e12 / tflops,
                         "peak_source": src}}


def sharded_parity(torch, dist, m, local, rank, world, dev):
    """Rank 0's all-reduced output of one sharded prefill (B2 x 300) and one decode step against the
    unsharded layer (all heads, the same weights) on the same GPU: max abs difference."""
    import torch.nn.functional as F
    H = W.SHAPE_QWEN.hidden_size
    g = torch.Generator(device=dev)
    g.manual_seed(11)
    x = torch.randn(2, 300, H, generator=g, device=dev).to(torch.bfloat16)
    xd = torch.randn(2, 1, H, generator=g, device=dev).to(torch.bfloat16)

    def layer_out(layer, lc, reduce):
        with torch.no_grad():
            S = torch.empty(2, lc.num_v_heads, lc.head_k_dim, lc.head_v_dim, device=dev)
            cs = torch.empty(2, lc.conv_dim, 3, dtype=torch.bfloat16, device=dev)
            cs2 = torch.empty_like(cs)
            mixed, z, bb, aa = layer.project(x)
            y = F.linear(layer.mixer(mixed, z, bb, aa, conv_state_out=cs, rec_state_out=S, token_by_token=False),
                         layer.out_proj.weight)
            mixed, z, bb, aa = layer.project(xd)
            yd = F.linear(layer.mixer(mixed, z, bb, aa, conv_state=cs, rec_state=S, conv_state_out=cs2,
                                      rec_state_out=S, token_by_token=True), layer.out_proj.weight)
            if reduce and world > 1:
                dist.all_reduce(y, op=dist.ReduceOp.SUM)
                dist.all_reduce(yd, op=dist.ReduceOp.SUM)
        return y.float(), yd.float()

    y, yd = layer_out(m, local, True)
    res = None
    if rank == 0:
        full, lfull = build_shard_layer(torch, 0, 1, dev)
        ry, ryd = layer_out(full, lfull, False)
        res = {"prefill_B2xT300_max_abs": float((y - ry).abs().max()), "decode_step_max_abs": float((yd - ryd).abs().max()),
               "reference": "the unsharded layer (all 32 value heads, same weights) on rank 0's GPU; outputs bf16"}
        del full
    torch.cuda.synchronize(dev)
    return res



def run_sharded_layer(torch, dist, m, local, rank, world, dev, barrier):
    """The value-head-sharded layer (this rank's heads, out_proj columns, one all-reduce): decode at
    the fixed global batch 64 (strong scaling) and at 64 per GPU (weak), prefill at the fixed global
    batch 8 x 8192 (strong) and 8 x 8192 per GPU (weak), and rank 0's output against the unsharded
    layer."""
    res = {"world": world,
           "layer": "head-sharded Gated DeltaNet layer: fused input projection of this rank's rows (cuBLAS), "
                    "token mixer on its 32/N value heads, out_proj column slice (cuBLAS), all-reduce (bf16 sum) "
                    "of the partial outputs: NCCL, and for decode also the one-shot NVLink peer kernel "
                    "(*_peer)"}
    res["decode_strong"] = sharded_decode(torch, dist, m, local, dev, world, barrier, 64)
    if world > 1:
        from visionstack_b200.peer import PeerAllReduce
        peer = PeerAllReduce(max_elems=64 * world * W.SHAPE_QWEN.hidden_size, nblocks=32, device=dev)
        res["decode_strong_peer"] = sharded_decode(torch, dist, m, local, dev, world, barrier, 64, peer=peer)
        res["decode_weak"] = sharded_decode(torch, dist, m, local, dev, world, barrier, 64 * world)
        res["decode_weak_peer"] = sharded_decode(torch, dist, m, local, dev, world, barrier, 64 * world, peer=peer)
        peer.close()
    res["prefill_strong"] = sharded_prefill(torch, dist, m, local, dev, world, barrier, 8, 8192)
    if world > 1:
        res["prefill_weak"] = sharded_prefill(torch, dist, m, local, dev, world, barrier, 8 * world, 8192)
    par = sharded_parity(torch, dist, m, local, rank, world, dev)
    if par is not None:
        res["parity_vs_unsharded"] = par
    torch.cuda.empty_cache()
    return res


def run_rollback(torch, dist, m, local, dev, world, barrier, steps=1024):
    """Speculative-decode verify with per-row rollback: batch 16, 4-token
    drafts, accepted counts uniform in 0..4 per row (numpy seed 5), each step =
    one verify launch (states after every draft token into the rows' free
    slots) + one accept launch (slot-table swap); ``steps`` steps in one CUDA
    graph."""
    from visionstack_b200 import StateSlots
    wl = W.WORKLOADS["rollback"]
    B, T = wl.batch * world, wl.seq_len  # global batch, 16 rows per GPU-equivalent
    hv, hk, d = local.num_v_heads, local.num_k_heads, local.head_k_dim
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    NIN = 16
    with torch.no_grad():
        x = torch.randn(NIN, B, T, W.SHAPE_QWEN.hidden_size, generator=g, device=dev).to(torch.bfloat16)
        ins = [m.project(x[i]) for i in range(NIN)]
        del x
    acc = torch.from_numpy(np.random.default_rng(wl.x_seed).integers(0, T + 1, size=(steps, B)).astype(np.int32))
    acc = acc.to(dev)
    slots = StateSlots(m, B, T, torch.bfloat16, dev)
    slots.load(torch.randn(B, local.conv_dim, 3, generator=g, device=dev).to(torch.bfloat16),
               0.02 * torch.randn(B, hv, d, d, generator=g, device=dev))
    out = torch.empty(B, T, local.value_dim, dtype=torch.bfloat16, device=dev)

    def step(i):
        mixed, z, bb, aa = ins[i % NIN]
        m.mixer_verify(mixed, z, bb, aa, slots, out=out)
        slots.accept(acc[i % steps])

    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        for i in range(4):
            step(i)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(steps):
            step(i)
    graph.replay()
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    with torch.cuda.stream(stream):
        ev0.record(stream)
        graph.replay()
        ev1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    t = torch.tensor([ev0.elapsed_time(ev1) / steps], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    del graph
    hbm, _, src = measured_peaks()
    nbytes = rollback_bytes(B, hk, hv, d, T)
    ach = nbytes / (ms * 1e-3) / 1e9
    return {"workload": f"speculative verify + rollback: B{B}, {T}-token drafts, accepted ~ U{{0..{T}}} (seed "
                        f"{wl.x_seed}), 16 k-heads / 32 v-heads (sharded), d128, bf16, {steps} steps",
            "steps_per_s": world * 1000.0 / ms, "unit": "B16 steps/s (whole job)", "ms_per_step": ms,
            "gpu_launches_per_step": 2,
            "roofline": {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm,
                         "peak_source": src, "bytes_per_step": nbytes,
                         "kernel": "gdn::dtma::decode_tma_kernel<128,8,bf16> with a slot table "
                                   "+ gdn::accept_slots_kernel"}}


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        local = int(os.environ.get("LOCAL_RANK", 0))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    try:
        run_ours(args, rank, world)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
