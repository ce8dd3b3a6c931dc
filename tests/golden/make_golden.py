"""Generate the golden fixtures by running the reference implementation.

Run where a checkout of the reference is available (read-only), given by
``--ref`` or the ``VISIONSTACK_REF`` environment variable:

    python tests/golden/make_golden.py --ref <reference checkout>

The reference is plain PyTorch, so it runs here on CPU.  Inputs come from
``numpy.random.default_rng`` seeds (``visionstack_b200.workloads``) so the
tests can regenerate the large ones instead of storing them; every fixture
stores a digest of its inputs so a drifting generator is caught.

Fixtures written next to this script:

* ``conv.npz``          causal conv continuation, fp32 and bf16 (gate3_models.py:1146-1167)
* ``solve.npz``         block triangular solve (gate3_models.py:1169-1191)
* ``delta.npz``         chunk / recurrent delta rule with checkpoints (gate3_models.py:1193-1245)
* ``layer_tiny_f32.npz``, ``layer_tiny_bf16.npz``  full layer with a hybrid cache:
                        prefill with checkpoints, decode steps, a 4-token verify step
* ``layer_cpu_plumbing.npz``  the B1 T256 fp32 layer + 16-token decode continuation
* ``cache.json``        checkpoint-position resolution of the hybrid cache and
                        the layer's state-dict names and shapes
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from visionstack_b200 import workloads as W  # noqa: E402


def digest(*arrays: np.ndarray) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a, dtype=np.float32).tobytes())
    return h.hexdigest()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("VISIONSTACK_REF"),
                    help="checkout of the reference (or set VISIONSTACK_REF)")
    args = ap.parse_args()
    if not args.ref:
        ap.error("give --ref <reference checkout> or set VISIONSTACK_REF")
    sys.path.insert(0, os.path.join(args.ref, "ShadowBoxer"))
    import torch

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    from models.qwen35.cache import Qwen3_5HybridCache
    from models.qwen35.config import Qwen3_5TextConfig
    from models.qwen35.deltanet import (
        Qwen3_5GatedDeltaNet,
        _causal_conv1d_fn,
        _chunk_gated_delta_rule,
        _recurrent_gated_delta_rule,
        _solve_unit_lower_triangular,
    )

    T_ = torch.from_numpy

    def npy(t):
        return t.detach().float().cpu().numpy()

    # ---------------- conv ----------------
    rng = np.random.default_rng(101)
    x = rng.standard_normal((1, 64, 16)).astype(np.float32)
    w = rng.standard_normal((64, 4)).astype(np.float32)
    full, full_state = _causal_conv1d_fn(T_(x), T_(w), activation="silu", return_final_state=True)
    pfx, mid = _causal_conv1d_fn(T_(x[:, :, :10]), T_(w), activation="silu", return_final_state=True)
    sfx, fin = _causal_conv1d_fn(T_(x[:, :, 10:]), T_(w), activation="silu", conv_state=mid,
                                 return_final_state=True)
    xb = W.round_bf16(rng.standard_normal((2, 96, 5)).astype(np.float32))
    wb = W.round_bf16(0.5 * rng.standard_normal((96, 4)).astype(np.float32))
    sb = W.round_bf16(rng.standard_normal((2, 96, 3)).astype(np.float32))
    bf = torch.bfloat16
    ob, stb = _causal_conv1d_fn(T_(xb).to(bf), T_(wb).to(bf), activation="silu", conv_state=T_(sb).to(bf),
                                return_final_state=True)
    x2 = xb[:, :, :2]
    o2, st2 = _causal_conv1d_fn(T_(x2).to(bf), T_(wb).to(bf), activation="silu", conv_state=T_(sb).to(bf),
                                return_final_state=True)
    o2n, st2n = _causal_conv1d_fn(T_(x2).to(bf), T_(wb).to(bf), activation="silu", return_final_state=True)
    np.savez_compressed(
        HERE / "conv.npz", x=x, w=w, full=npy(full), full_state=npy(full_state), pfx=npy(pfx), mid=npy(mid),
        sfx=npy(sfx), fin=npy(fin), xb=xb, wb=wb, sb=sb, ob=npy(ob), stb=npy(stb), o2=npy(o2), st2=npy(st2),
        o2n=npy(o2n), st2n=npy(st2n))

    # ---------------- triangular solve ----------------
    rng = np.random.default_rng(102)
    out = {}
    for n in (16, 20, 32, 64):
        ut = (np.tril(rng.standard_normal((1, 2, 1, n, n)).astype(np.float32), -1) * 0.05
              + np.eye(n, dtype=np.float32))
        rhs = rng.standard_normal((1, 2, 1, n, 48)).astype(np.float32)
        out[f"ut{n}"] = ut
        out[f"rhs{n}"] = rhs
        out[f"sol{n}"] = npy(_solve_unit_lower_triangular(T_(ut), T_(rhs)))
    np.savez_compressed(HERE / "solve.npz", **out)

    # ---------------- delta rule ----------------
    rng = np.random.default_rng(103)
    d = {}

    def gates(B, T, H):
        g = (-rng.random((B, T, H)) * 0.25).astype(np.float32)
        b = (1.0 / (1.0 + np.exp(-rng.standard_normal((B, T, H))))).astype(np.float32)
        return g, b

    q = rng.standard_normal((1, 20, 4, 32)).astype(np.float32)
    k = rng.standard_normal((1, 20, 4, 32)).astype(np.float32)
    v = rng.standard_normal((1, 20, 4, 32)).astype(np.float32)
    g, b = gates(1, 20, 4)
    cps = {}
    o_full = _chunk_gated_delta_rule(T_(q), T_(k), T_(v), T_(g), T_(b), output_final_state=False,
                                     checkpoint_positions=[12, 16], checkpoint_states_out=cps)
    o_rec, s_rec = _recurrent_gated_delta_rule(T_(q), T_(k), T_(v), T_(g), T_(b), output_final_state=True)
    d.update(a_q=q, a_k=k, a_v=v, a_g=g, a_b=b, a_out=npy(o_full), a_cp12=npy(cps[12]), a_cp16=npy(cps[16]),
             a_rec_out=npy(o_rec), a_rec_state=npy(s_rec))
    # longer: several chunks of 64 + padding, initial state, sub-chunk and boundary checkpoints
    B, T, H, D = 2, 150, 4, 32
    q = rng.standard_normal((B, T, H, D)).astype(np.float32)
    k = rng.standard_normal((B, T, H, D)).astype(np.float32)
    v = rng.standard_normal((B, T, H, D)).astype(np.float32)
    g, b = W.make_gate_inputs(rng, B, T, H)
    s0 = (0.1 * rng.standard_normal((B, H, D, D))).astype(np.float32)
    cps = {}
    cp_list = [40, 45, 100, 128, 163, 190, 300]
    o, s = _chunk_gated_delta_rule(T_(q), T_(k), T_(v), T_(g), T_(b), initial_state=T_(s0), output_final_state=True,
                                   checkpoint_positions=cp_list, checkpoint_states_out=cps, past_seen_tokens=40)
    d.update(b_q=q, b_k=k, b_v=v, b_g=g, b_b=b, b_s0=s0, b_out=npy(o), b_state=npy(s),
             b_cp_keys=np.array(sorted(cps), dtype=np.int64),
             b_cp_vals=np.stack([npy(cps[c]) for c in sorted(cps)]))
    # T <= 8 with a state takes the token-by-token path, with per-token checkpoints
    T = 5
    q5, k5, v5 = (rng.standard_normal((B, T, H, D)).astype(np.float32) for _ in range(3))
    g5, b5 = W.make_gate_inputs(rng, B, T, H)
    cps = {}
    o, s = _chunk_gated_delta_rule(T_(q5), T_(k5), T_(v5), T_(g5), T_(b5), initial_state=T_(s0),
                                   output_final_state=True, checkpoint_positions=[8, 9, 10, 12],
                                   checkpoint_states_out=cps, past_seen_tokens=7)
    d.update(c_q=q5, c_k=k5, c_v=v5, c_g=g5, c_b=b5, c_out=npy(o), c_state=npy(s),
             c_cp_keys=np.array(sorted(cps), dtype=np.int64),
             c_cp_vals=np.stack([npy(cps[c]) for c in sorted(cps)]))
    # T = 3 without a state: chunk path with chunk 16 and zero padding
    o, s = _chunk_gated_delta_rule(T_(q5[:, :3]), T_(k5[:, :3]), T_(v5[:, :3]), T_(g5[:, :3]), T_(b5[:, :3]),
                                   output_final_state=True)
    d.update(e_out=npy(o), e_state=npy(s))
    np.savez_compressed(HERE / "delta.npz", **d)

    # ---------------- layers ----------------
    def make_module(shape, params, dtype):
        cfg = Qwen3_5TextConfig(
            hidden_size=shape.hidden_size, linear_num_key_heads=shape.num_k_heads,
            linear_num_value_heads=shape.num_v_heads, linear_key_head_dim=shape.head_k_dim,
            linear_value_head_dim=shape.head_v_dim, linear_conv_kernel_dim=shape.conv_kernel,
            rms_norm_eps=shape.rms_norm_eps, num_hidden_layers=4)
        m = Qwen3_5GatedDeltaNet(cfg, 0)
        tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
        m = m.to(tdt)
        sd = {}
        for name, arr in params.items():
            t = T_(arr)
            sd[name] = t if name in ("A_log", "dt_bias") else t.to(tdt)
        for name, p in m.named_parameters():
            p.data = sd[name].clone()
        return m.eval(), tdt

    def layer_case(shape, dtype, tag):
        wl = W.Workload(tag, shape, 2, 80, 3, dtype, 11, 12)
        params = W.make_layer_params(shape, wl.w_seed, dtype)
        m, tdt = make_module(shape, params, dtype)
        res = {f"p_{k}": v for k, v in params.items()}
        x = W.make_hidden(wl)
        mask = np.ones((2, 80), dtype=np.float32)
        mask[1, :5] = 0.0
        res["x"] = x
        res["mask"] = mask
        with torch.inference_mode():
            # no cache
            y0 = m(T_(x).to(tdt), attention_mask=T_(mask).to(torch.long))
            res["y_nocache"] = npy(y0)
            cache = Qwen3_5HybridCache(record_checkpoints=True, checkpoint_positions=[3, 16, 45, 64, 80])
            cache.resolve_active_checkpoints(0, 80)
            y1 = m(T_(x).to(tdt), cache=cache)
            cache.past_seen_tokens = 80
            res["y_prefill"] = npy(y1)
            res["conv_state_prefill"] = npy(cache.conv_states[0])
            res["rec_state_prefill"] = npy(cache.recurrent_states[0])
            cks = sorted(cache.recurrent_checkpoints)
            res["cp_keys"] = np.array(cks, dtype=np.int64)
            res["cp_rec"] = np.stack([npy(cache.recurrent_checkpoints[c][0]) for c in cks])
            res["cp_conv"] = np.stack([npy(cache.conv_checkpoints[c][0]) for c in cks])
            cache.record_checkpoints = False
            ys = []
            for t in range(3):
                xt = W.make_hidden(wl, seq_len=1, seed_offset=t + 1)
                res[f"x_dec{t}"] = xt
                ys.append(npy(m(T_(xt).to(tdt), cache=cache)))
                cache.past_seen_tokens += 1
            res["y_dec"] = np.concatenate(ys, axis=1)
            res["conv_state_dec"] = npy(cache.conv_states[0])
            res["rec_state_dec"] = npy(cache.recurrent_states[0])
            # 4-token verify step with per-token checkpoints (T <= 8 path)
            ver = cache.clone_and_expand(1, record_checkpoints=True, checkpoint_positions=[84, 85, 86, 87])
            ver.resolve_active_checkpoints(83, 4)
            xv = W.make_hidden(wl, seq_len=4, seed_offset=9)
            res["x_ver"] = xv
            res["y_ver"] = npy(m(T_(xv).to(tdt), cache=ver))
            cks = sorted(ver.recurrent_checkpoints)
            res["ver_cp_keys"] = np.array(cks, dtype=np.int64)
            res["ver_cp_rec"] = np.stack([npy(ver.recurrent_checkpoints[c][0]) for c in cks])
            res["ver_cp_conv"] = np.stack([npy(ver.conv_checkpoints[c][0]) for c in cks])
            res["ver_rec_state"] = npy(ver.recurrent_states[0])
            res["ver_conv_state"] = npy(ver.conv_states[0])
        np.savez_compressed(HERE / f"layer_{tag}.npz", **res)

    layer_case(W.SHAPE_TINY, "f32", "tiny_f32")
    layer_case(W.SHAPE_TINY, "bf16", "tiny_bf16")

    # the B1 T256 fp32 layer and its 16-token decode continuation
    wl = W.WORKLOADS["cpu_plumbing"]
    params = W.make_layer_params(wl.shape, wl.w_seed, wl.dtype)
    m, tdt = make_module(wl.shape, params, wl.dtype)
    x = W.make_hidden(wl)
    res = {"input_digest": np.frombuffer(bytes.fromhex(digest(x, *[params[k] for k in sorted(params)])),
                                         dtype=np.uint8)}
    with torch.inference_mode():
        cache = Qwen3_5HybridCache()
        y = m(T_(x), cache=cache)
        cache.past_seen_tokens = wl.seq_len
        res["y_prefill"] = npy(y)
        res["rec_state_prefill"] = npy(cache.recurrent_states[0])
        res["conv_state_prefill"] = npy(cache.conv_states[0])
        ys = []
        for t in range(wl.steps):
            xt = W.make_hidden(wl, seq_len=1, seed_offset=t + 1)
            ys.append(npy(m(T_(xt), cache=cache)))
            cache.past_seen_tokens += 1
        res["y_dec"] = np.concatenate(ys, axis=1)
        res["rec_state_dec"] = npy(cache.recurrent_states[0])
        res["conv_state_dec"] = npy(cache.conv_states[0])
    np.savez_compressed(HERE / "layer_cpu_plumbing.npz", **res)

    # ---------------- hybrid-cache checkpoint resolution ----------------
    cases = []
    for (past, T, min_tok, structural, requested) in [
        (0, 53, 4, [21, 33], None), (0, 256, 0, [], None), (100, 1, 0, [], None), (0, 9, 0, [], None),
        (0, 8192, 0, [500, 1000], None), (37, 300, 60, [40, 64, 200], None), (0, 80, 0, [], [16, 48, 64, 80]),
        (83, 4, 0, [], [84, 85, 86, 87]), (10, 5, 12, [], [11, 12, 13, 15, 99]),
    ]:
        c = Qwen3_5HybridCache(record_checkpoints=True, checkpoint_positions=requested,
                               min_checkpoint_token=min_tok, structural_checkpoints=structural)
        cases.append({"past": past, "T": T, "min_tok": min_tok, "structural": structural,
                      "requested": requested, "result": c.resolve_active_checkpoints(past, T)})
    token_lists = [
        [248045, 872, 198, 248053] + [248056] * 16 + [248054] + list(range(200, 260)) + [248044],
        [248045, 872, 198] + list(range(101, 121)) + [248044],
        list(range(1000, 1300)),
        [248046, 5, 6] + list(range(10, 80)) + [248044, 3, 4],
    ]
    structural = []
    for toks in token_lists:
        ms, cps = Qwen3_5HybridCache.derive_structural_checkpoints(toks)
        structural.append({"tokens": toks, "min_snap": ms, "cps": cps})
    ref_layer = Qwen3_5GatedDeltaNet(Qwen3_5TextConfig(hidden_size=2048), 3)
    state_dict = {k: list(v.shape) for k, v in ref_layer.state_dict().items()}
    with open(HERE / "cache.json", "w") as f:
        json.dump({"resolve": cases, "structural": structural, "state_dict": state_dict}, f, indent=1)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
