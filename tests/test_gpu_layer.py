"""The drop-in layer and the functional boundary on the GPU against the
reference's own outputs (golden fixtures) and the reference's self-test
properties (ShadowBoxer/sanitycheck/gate3_models.py:1146-1276)."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from tests.helpers import (assert_bf16_close, assert_f32_close, assert_state_close, max_abs, rel_max, to_np)
from tests.test_gpu_mixer import TDT, make_layer
from visionstack_b200 import (Qwen3_5GatedDeltaNet, Qwen3_5HybridCache, Qwen3_5TextConfig, _causal_conv1d_fn,
                              _chunk_gated_delta_rule, _recurrent_gated_delta_rule)
from visionstack_b200 import workloads as W

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    return np.load(os.path.join(GOLD, name))


def cu(a, dt=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda().to(dt)


def layer_from_fixture(d, shape, dtype):
    cfg = Qwen3_5TextConfig(hidden_size=shape.hidden_size, linear_num_key_heads=shape.num_k_heads,
                            linear_num_value_heads=shape.num_v_heads, linear_key_head_dim=shape.head_k_dim,
                            linear_value_head_dim=shape.head_v_dim, rms_norm_eps=shape.rms_norm_eps,
                            num_hidden_layers=4)
    m = Qwen3_5GatedDeltaNet(cfg, 0)
    with torch.no_grad():
        for name, p in m.named_parameters():
            t = torch.from_numpy(d["p_" + name])
            p.data = t if name in ("A_log", "dt_bias") else t.to(TDT[dtype])
    return m.cuda()


def out_close(ours, ref, dtype, what, f32_tol=1e-4):
    if dtype == "bf16":
        assert_bf16_close(ours, ref, what)
    else:
        assert_f32_close(ours, ref, f32_tol, what)


def conv_close(ours, ref, dtype, what):
    # layer-level conv states are copies of the projection GEMM output, whose
    # last-bit rounding is cuBLAS's here and CPU BLAS's in the fixture
    o, r = to_np(ours), to_np(ref)
    if dtype == "bf16":
        assert np.mean(o == r) > 0.99 and max_abs(o, r) <= 2.0 ** -7 * max(1.0, float(np.abs(r).max())), what
    else:
        assert max_abs(o, r) < 1e-5, what


@pytest.mark.parametrize("tag,dtype", [("tiny_f32", "f32"), ("tiny_bf16", "bf16")])
def test_layer_cache_trajectory_vs_reference(tag, dtype):
    d = load(f"layer_{tag}.npz")
    m = layer_from_fixture(d, W.SHAPE_TINY, dtype)
    dt = TDT[dtype]
    with torch.inference_mode():
        y0 = m(cu(d["x"], dt), attention_mask=cu(d["mask"]).long())
        out_close(y0, d["y_nocache"], dtype, "no cache + mask")
        cache = Qwen3_5HybridCache(record_checkpoints=True, checkpoint_positions=[3, 16, 45, 64, 80])
        cache.resolve_active_checkpoints(0, 80)
        y1 = m(cu(d["x"], dt), cache=cache)
        cache.past_seen_tokens = 80
        out_close(y1, d["y_prefill"], dtype, "prefill")
        conv_close(cache.conv_states[0], d["conv_state_prefill"], dtype, "conv state")
        assert cache.recurrent_states[0].dtype == torch.float32
        assert_state_close(cache.recurrent_states[0], d["rec_state_prefill"], "prefill state")
        assert sorted(cache.recurrent_checkpoints) == list(d["cp_keys"]) == sorted(cache.conv_checkpoints)
        for i, c in enumerate(d["cp_keys"]):
            conv_close(cache.conv_checkpoints[int(c)][0], d["cp_conv"][i], dtype, f"conv cp {c}")
            assert_state_close(cache.recurrent_checkpoints[int(c)][0], d["cp_rec"][i], f"cp {c}")
        cache.record_checkpoints = False
        ys = []
        for t in range(3):
            ys.append(m(cu(d[f"x_dec{t}"], dt), cache=cache))
            cache.past_seen_tokens += 1
        out_close(torch.cat(ys, 1), d["y_dec"], dtype, "decode")
        assert_state_close(cache.recurrent_states[0], d["rec_state_dec"], "decode state")
        ver = cache.clone_and_expand(1, record_checkpoints=True, checkpoint_positions=[84, 85, 86, 87])
        ver.resolve_active_checkpoints(83, 4)
        yv = m(cu(d["x_ver"], dt), cache=ver)
        out_close(yv, d["y_ver"], dtype, "verify")
        assert sorted(ver.recurrent_checkpoints) == list(d["ver_cp_keys"]) == [84, 85, 86, 87]
        for i, c in enumerate(d["ver_cp_keys"]):
            conv_close(ver.conv_checkpoints[int(c)][0], d["ver_cp_conv"][i], dtype, f"verify conv cp {c}")
            assert_state_close(ver.recurrent_checkpoints[int(c)][0], d["ver_cp_rec"][i], f"verify cp {c}")
        assert_state_close(ver.recurrent_states[0], d["ver_rec_state"], "verify state")


def test_layer_cpu_plumbing_config_vs_reference():
    """B1 T256 hidden 1024 fp32 layer + 16-token decode continuation."""
    d = load("layer_cpu_plumbing.npz")
    wl = W.WORKLOADS["cpu_plumbing"]
    m, _ = make_layer(wl.shape, "f32", seed=wl.w_seed)
    with torch.inference_mode():
        cache = Qwen3_5HybridCache()
        y = m(cu(W.make_hidden(wl)), cache=cache)
        cache.past_seen_tokens = wl.seq_len
        assert_f32_close(y, d["y_prefill"], 1e-4, "prefill")
        assert_state_close(cache.recurrent_states[0], d["rec_state_prefill"], "prefill state", tol=1e-4)
        ys = []
        for t in range(wl.steps):
            ys.append(m(cu(W.make_hidden(wl, 1, t + 1)), cache=cache))
            cache.past_seen_tokens += 1
        assert_f32_close(torch.cat(ys, 1), d["y_dec"], 1e-4, "decode")
        assert_state_close(cache.recurrent_states[0], d["rec_state_dec"], "decode state", tol=1e-4)


def test_trajectory_splice_property():
    """gate3_models.py:1247-1276 on one layer: a checkpoint recorded during an
    80-token pass, extracted and continued, reproduces the unsplit pass."""
    shape = W.SHAPE_TINY
    m, _ = make_layer(shape, "bf16", seed=7)
    x = cu(W.make_hidden(W.Workload("s", shape, 1, 80, 1, "bf16", 21, 7)), torch.bfloat16)
    with torch.inference_mode():
        c = Qwen3_5HybridCache(record_checkpoints=True, checkpoint_positions=[16, 48, 64])
        c.resolve_active_checkpoints(0, 80)
        full = m(x, cache=c)
        c.past_seen_tokens = 80
        cp = c.extract_checkpoint(64)
        tail = m(x[:, 64:], cache=cp)
    spliced = torch.cat([full[:, :64], tail], 1)
    assert max_abs(full, spliced) <= 0.0625 and float((full - spliced).abs().float().mean()) < 2e-3


def test_inplace_ownership_rules():
    shape = W.SHAPE_TINY
    m, _ = make_layer(shape, "bf16")
    x = cu(np.random.default_rng(0).standard_normal((2, 1, shape.hidden_size)).astype(np.float32), torch.bfloat16)
    with torch.inference_mode():
        c = Qwen3_5HybridCache()
        c.recurrent_states[0] = torch.randn(2, 4, 32, 32, device="cuda")
        foreign = c.recurrent_states[0]
        keep = foreign.clone()
        m(x, cache=c)  # foreign state: never written
        assert torch.equal(foreign, keep) and c.recurrent_states[0] is not foreign
        mine = c.recurrent_states[0]
        m(x, cache=c)  # our own state: updated in place
        assert c.recurrent_states[0] is mine
        m.inplace_state = False
        m(x, cache=c)
        assert c.recurrent_states[0] is not mine


# ---------------- functional boundary vs the reference's fixtures ----------------

def test_functional_conv_continuation():
    d = load("conv.npz")
    full, st = _causal_conv1d_fn(cu(d["x"]), cu(d["w"]), activation="silu", return_final_state=True)
    assert max_abs(full, d["full"]) < 1e-6 and max_abs(st, d["full_state"]) == 0.0
    pfx, mid = _causal_conv1d_fn(cu(d["x"][:, :, :10]), cu(d["w"]), activation="silu", return_final_state=True)
    sfx, fin = _causal_conv1d_fn(cu(d["x"][:, :, 10:]), cu(d["w"]), activation="silu", conv_state=mid,
                                 return_final_state=True)
    assert max_abs(torch.cat([pfx, sfx], -1), full) < 1e-6 and max_abs(fin, d["fin"]) == 0.0
    bf = torch.bfloat16
    ob, stb = _causal_conv1d_fn(cu(d["xb"], bf), cu(d["wb"], bf), activation="silu", conv_state=cu(d["sb"], bf),
                                return_final_state=True)
    assert max_abs(stb, d["stb"]) == 0.0
    assert np.mean(to_np(ob) == d["ob"]) > 0.99


def test_functional_delta_rule_checkpoints():
    d = load("delta.npz")
    cps = {}
    out = _chunk_gated_delta_rule(cu(d["a_q"]), cu(d["a_k"]), cu(d["a_v"]), cu(d["a_g"]), cu(d["a_b"]),
                                  checkpoint_positions=[12, 16], checkpoint_states_out=cps)
    assert max_abs(out, d["a_out"]) < 1e-5
    assert max_abs(cps[12], d["a_cp12"]) < 1e-5 and max_abs(cps[16], d["a_cp16"]) < 1e-5
    o, s = _recurrent_gated_delta_rule(cu(d["a_q"]), cu(d["a_k"]), cu(d["a_v"]), cu(d["a_g"]), cu(d["a_b"]),
                                       output_final_state=True)
    assert max_abs(o, d["a_rec_out"]) < 1e-5 and max_abs(s, d["a_rec_state"]) < 1e-5
    cps = {}
    o, s = _chunk_gated_delta_rule(cu(d["b_q"]), cu(d["b_k"]), cu(d["b_v"]), cu(d["b_g"]), cu(d["b_b"]),
                                   initial_state=cu(d["b_s0"]), output_final_state=True,
                                   checkpoint_positions=[40, 45, 100, 128, 163, 190, 300],
                                   checkpoint_states_out=cps, past_seen_tokens=40)
    assert max_abs(o, d["b_out"]) < 2e-5 and rel_max(s, d["b_state"]) < 1e-5
    assert sorted(cps) == list(d["b_cp_keys"])
    for i, c in enumerate(sorted(cps)):
        assert rel_max(cps[c], d["b_cp_vals"][i]) < 1e-5
    cps = {}
    o, s = _chunk_gated_delta_rule(cu(d["c_q"]), cu(d["c_k"]), cu(d["c_v"]), cu(d["c_g"]), cu(d["c_b"]),
                                   initial_state=cu(d["b_s0"]), output_final_state=True,
                                   checkpoint_positions=[8, 9, 10, 12], checkpoint_states_out=cps,
                                   past_seen_tokens=7)
    assert max_abs(o, d["c_out"]) < 1e-5 and rel_max(s, d["c_state"]) < 1e-5
    assert sorted(cps) == [8, 9, 10, 12]
    o, s = _chunk_gated_delta_rule(cu(d["c_q"][:, :3]), cu(d["c_k"][:, :3]), cu(d["c_v"][:, :3]),
                                   cu(d["c_g"][:, :3]), cu(d["c_b"][:, :3]), output_final_state=True)
    assert max_abs(o, d["e_out"]) < 1e-5 and rel_max(s, d["e_state"]) < 1e-5


def test_fused_input_projection():
    """The four input projections run as one GEMM over a fused weight whose row ranges the
    parameters become: the state dict keeps its names, shapes and values, loading a state dict
    afterwards updates the fused weight, and the layer output matches the four separate GEMMs."""
    shape = W.SHAPE_SMALL
    m, _ = make_layer(shape, "bf16")
    sd_before = {k: v.clone() for k, v in m.state_dict().items()}
    g = torch.Generator(device="cuda")
    g.manual_seed(21)
    x = torch.randn(2, 70, shape.hidden_size, generator=g, device="cuda").to(torch.bfloat16)
    with torch.no_grad():
        fused = m.project(x)
        f = m._in_proj_fused
        assert f is not None and m.in_proj_z.weight.data_ptr() == f[shape.conv_dim].data_ptr()
        sd_after = m.state_dict()
        assert list(sd_after) == list(sd_before)
        for k in sd_before:
            assert sd_after[k].shape == sd_before[k].shape and torch.equal(sd_after[k], sd_before[k]), k
        m.fuse_in_proj = False
        sep = m.project(x)
        for a, b in zip(fused, sep):
            assert a.shape == b.shape
            assert (a.float() - b.float()).abs().max().item() <= 0.02 * b.float().abs().max().item() + 1e-2
        y_sep = m(x)
        m.fuse_in_proj = True
        y_fused = m(x)
        assert_bf16_close(y_fused, y_sep, "layer output, fused vs separate projections", scale=2.0)
        # loading a state dict after the fusion writes through to the fused weight
        sd2 = {k: (v * 0.5 if k == "in_proj_b.weight" else v) for k, v in sd_before.items()}
        m.load_state_dict(sd2)
        assert m.project(x)[2].data_ptr() != 0
        assert torch.equal(m._in_proj_fused[shape.conv_dim + shape.value_dim:
                                            shape.conv_dim + shape.value_dim + shape.num_v_heads],
                           sd2["in_proj_b.weight"])
