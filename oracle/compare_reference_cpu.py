"""Speed of the numpy oracle port against the reference's own PyTorch CPU code.

The timed CPU baseline of ``bench.py`` runs the oracle (``oracle/gdn_oracle.py``, a
restatement of ShadowBoxer/models/qwen35/deltanet.py), because the reference cannot
travel to the GPU box.  This script, run where the reference checkout is available,
times both on the same inputs and the same thread counts and prints the factor
(oracle time / reference time) per workload, so that a port rate measured on the
GPU box translates into the reference's rate:

* decode: one token-by-token delta-rule step at B64 x 32 value heads, d 128
  (``_recurrent_gated_delta_rule``, deltanet.py:165-233), fp32 operands;
* prefill: the chunked delta rule on 8 rows x 1024 tokens x 32 value heads
  (``_chunk_gated_delta_rule``, deltanet.py:236-407), fp32 operands;

the reference with torch's intra-op threads, the oracle with its batch rows split over the
same number of host threads, as bench.py runs it;
* layer: the reference's CPU-runnable layer case (B1 x 256 tokens, hidden 1024,
  8 / 8 heads of 128, fp32) through the full layer forward with a hybrid cache,
  then 16 single-token steps (deltanet.py:447-563 against the oracle's
  ``deltanet_layer_forward``).

Usage:  python oracle/compare_reference_cpu.py --ref <reference checkout> [--threads N]
(or set VISIONSTACK_REF).  Test infrastructure only: nothing in the package imports it.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(REPO))

from oracle import gdn_oracle as O  # noqa: E402
from visionstack_b200 import workloads as W  # noqa: E402


def _best(fn, reps: int) -> float:
    fn()
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    return float(np.median(ts))


def _delta_inputs(B, T, H, d, seed):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, T, H, d)).astype(np.float32)
    k = rng.standard_normal((B, T, H, d)).astype(np.float32)
    v = rng.standard_normal((B, T, H, d)).astype(np.float32)
    g = -np.abs(rng.standard_normal((B, T, H))).astype(np.float32) * 0.1
    beta = (1.0 / (1.0 + np.exp(-rng.standard_normal((B, T, H))))).astype(np.float32)
    S0 = (0.02 * rng.standard_normal((B, H, d, d))).astype(np.float32)
    return q, k, v, g, beta, S0


def _split_rows(fn, rows: int, threads: int) -> None:
    """fn(r0, r1) over `threads` contiguous row slices on host threads, BLAS held to one thread
    per slice (the way bench.py's CPU baseline runs the oracle)."""
    from concurrent.futures import ThreadPoolExecutor

    from threadpoolctl import threadpool_limits
    P = max(1, min(threads, rows))
    cut = [rows * i // P for i in range(P + 1)]
    if P == 1:
        fn(0, rows)
        return
    with threadpool_limits(limits=1, user_api="blas"), ThreadPoolExecutor(P) as ex:
        list(ex.map(lambda i: fn(cut[i], cut[i + 1]), range(P)))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("VISIONSTACK_REF"),
                    help="checkout of the reference (or set VISIONSTACK_REF)")
    ap.add_argument("--threads", type=int, default=len(os.sched_getaffinity(0)))
    ap.add_argument("--reps", type=int, default=3)
    args = ap.parse_args()
    if not args.ref:
        ap.error("give --ref <reference checkout> or set VISIONSTACK_REF")
    sys.path.insert(0, os.path.join(args.ref, "ShadowBoxer"))
    import torch
    from threadpoolctl import threadpool_limits

    from models.qwen35 import deltanet as R
    from models.qwen35.cache import Qwen3_5HybridCache
    from models.qwen35.config import Qwen3_5TextConfig

    results = {}
    for threads in sorted({1, args.threads}):
        torch.set_num_threads(threads)
        row = {}
        with threadpool_limits(limits=threads, user_api="blas"), torch.inference_mode():
            # decode step, B64 x 32 heads
            q, k, v, g, beta, S0 = _delta_inputs(64, 1, 32, 128, 1)
            tq, tk, tv, tg, tb, tS = (torch.from_numpy(a) for a in (q, k, v, g, beta, S0))
            t_ref = _best(lambda: R._recurrent_gated_delta_rule(tq, tk, tv, tg, tb, initial_state=tS,
                                                                output_final_state=True), args.reps)
            # the oracle as bench.py runs it: the batch rows split over `threads` host threads
            t_or = _best(lambda: _split_rows(lambda r0, r1: O.recurrent_gated_delta_rule(
                q[r0:r1], k[r0:r1], v[r0:r1], g[r0:r1], beta[r0:r1], initial_state=S0[r0:r1],
                output_final_state=True), 64, threads), args.reps)
            row["decode_B64"] = {"reference_s": t_ref, "oracle_s": t_or, "oracle_over_reference": t_or / t_ref}
            # chunked prefill, 8 rows x 1024 tokens x 32 heads (one row per oracle thread)
            q, k, v, g, beta, S0 = _delta_inputs(8, 1024, 32, 128, 2)
            tq, tk, tv, tg, tb = (torch.from_numpy(a) for a in (q, k, v, g, beta))
            t_ref = _best(lambda: R._chunk_gated_delta_rule(tq, tk, tv, tg, tb, output_final_state=True), args.reps)
            t_or = _best(lambda: _split_rows(lambda r0, r1: O.chunk_gated_delta_rule(
                q[r0:r1], k[r0:r1], v[r0:r1], g[r0:r1], beta[r0:r1], output_final_state=True), 8, threads), args.reps)
            row["prefill_8x1024"] = {"reference_s": t_ref, "oracle_s": t_or, "oracle_over_reference": t_or / t_ref}
            # the CPU-runnable layer case: B1 x 256 fp32, then 16 steps
            wl = W.WORKLOADS["cpu_plumbing"]
            s = wl.shape
            p = W.make_layer_params(s, wl.w_seed, "f32")
            cfg = Qwen3_5TextConfig(hidden_size=s.hidden_size, linear_num_key_heads=s.num_k_heads,
                                    linear_num_value_heads=s.num_v_heads, linear_key_head_dim=s.head_k_dim,
                                    linear_value_head_dim=s.head_v_dim, linear_conv_kernel_dim=s.conv_kernel,
                                    rms_norm_eps=s.rms_norm_eps, num_hidden_layers=4)
            layer = R.Qwen3_5GatedDeltaNet(cfg, 0).float().eval()
            layer.load_state_dict({kk: torch.from_numpy(np.ascontiguousarray(vv)).float() for kk, vv in p.items()})
            x = torch.from_numpy(W.make_hidden(wl))
            xs = [torch.from_numpy(W.make_hidden(wl, seq_len=1, seed_offset=i + 1)) for i in range(16)]

            def ref_layer():
                c = Qwen3_5HybridCache()
                layer(x, cache=c)
                c.past_seen_tokens = wl.seq_len
                for xd in xs:
                    layer(xd, cache=c)
                    c.past_seen_tokens += 1

            def oracle_layer():
                c = O.OracleCache()
                O.deltanet_layer_forward(p, s, x.numpy(), "f32", cache=c)
                c.past_seen_tokens = wl.seq_len
                for xd in xs:
                    O.deltanet_layer_forward(p, s, xd.numpy(), "f32", cache=c)
                    c.past_seen_tokens += 1

            t_ref = _best(ref_layer, args.reps)
            t_or = _best(oracle_layer, args.reps)
            row["layer_B1xT256_plus_16_steps"] = {"reference_s": t_ref, "oracle_s": t_or,
                                                  "oracle_over_reference": t_or / t_ref}
        results[f"threads_{threads}"] = row
    print(json.dumps({"host_cpus": len(os.sched_getaffinity(0)), "torch": torch.__version__,
                      "numpy": np.__version__, "results": results}, indent=1))


if __name__ == "__main__":
    main()
