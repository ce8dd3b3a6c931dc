"""Parity of the fused token-mixer kernels (through the C ABI) with the
numpy oracle on identical seeded projection outputs."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gdn_oracle as O
from tests.helpers import (assert_bf16_close, assert_bit_exact, assert_f32_close, assert_state_close, to_np)
from visionstack_b200 import Qwen3_5GatedDeltaNet, Qwen3_5TextConfig
from visionstack_b200 import workloads as W

pytestmark = pytest.mark.gpu

TDT = {"bf16": torch.bfloat16, "f32": torch.float32}


def make_layer(shape: W.LayerShape, dtype: str, seed: int = 1):
    cfg = Qwen3_5TextConfig(hidden_size=shape.hidden_size, linear_num_key_heads=shape.num_k_heads,
                            linear_num_value_heads=shape.num_v_heads, linear_key_head_dim=shape.head_k_dim,
                            linear_value_head_dim=shape.head_v_dim, linear_conv_kernel_dim=shape.conv_kernel,
                            rms_norm_eps=shape.rms_norm_eps)
    m = Qwen3_5GatedDeltaNet(cfg, 0)
    params = W.make_layer_params(shape, seed, dtype)
    with torch.no_grad():
        for name, p in m.named_parameters():
            t = torch.from_numpy(params[name])
            p.data = t if name in ("A_log", "dt_bias") else t.to(TDT[dtype])
    return m.cuda(), params


def mixer_inputs(shape: W.LayerShape, B: int, T: int, dtype: str, seed: int, with_state: bool):
    rng = np.random.default_rng(seed)
    f = lambda *s, sc=1.0: W.cast(sc * rng.standard_normal(s).astype(np.float32), dtype)  # noqa: E731
    d = {
        "mixed": f(B, T, shape.conv_dim, sc=0.7),
        "z": f(B, T, shape.value_dim, sc=0.7),
        "b": f(B, T, shape.num_v_heads, sc=1.4),
        "a": f(B, T, shape.num_v_heads, sc=1.4),
    }
    if with_state:
        d["conv_state"] = f(B, shape.conv_dim, shape.conv_kernel - 1, sc=0.7)
        d["rec_state"] = (0.05 * rng.standard_normal(
            (B, shape.num_v_heads, shape.head_k_dim, shape.head_v_dim))).astype(np.float32)
    return d


def run_ours(m, shape, d, dtype, token_by_token, offsets=(), register_kernel=False, fused_prefill=False,
             prep_in_kernel_prefill=False):
    dev = torch.device("cuda")
    t = lambda a: torch.from_numpy(a).to(dev).to(TDT[dtype])  # noqa: E731
    B, T = d["mixed"].shape[:2]
    L = shape.conv_kernel - 1
    cs = t(d["conv_state"]) if "conv_state" in d else None
    rs = torch.from_numpy(d["rec_state"]).to(dev) if "rec_state" in d else None
    cs_out = torch.empty((B, shape.conv_dim, L), dtype=TDT[dtype], device=dev)
    rs_out = torch.empty((B, shape.num_v_heads, shape.head_k_dim, shape.head_v_dim), device=dev)
    n = len(offsets)
    st_ck = torch.full((n, B, shape.num_v_heads, shape.head_k_dim, shape.head_v_dim), float("nan"),
                       device=dev) if n else None
    cv_ck = torch.zeros((n, B, shape.conv_dim, L), dtype=TDT[dtype], device=dev) if n else None
    out = m.mixer(t(d["mixed"]), t(d["z"]), t(d["b"]), t(d["a"]), conv_state=cs, rec_state=rs,
                  conv_state_out=cs_out, rec_state_out=rs_out, checkpoint_offsets=offsets,
                  state_checkpoints=st_ck, conv_checkpoints=cv_ck, token_by_token=token_by_token,
                  register_kernel=register_kernel, fused_prefill=fused_prefill,
                  prep_in_kernel_prefill=prep_in_kernel_prefill)
    torch.cuda.synchronize()
    return out, cs_out, rs_out, st_ck, cv_ck


def run_oracle(shape, params, d, dtype, chunk, offsets=()):
    B, T = d["mixed"].shape[:2]
    return O.mixer_forward(shape, d["mixed"], d["z"].reshape(B, T, shape.num_v_heads, shape.head_v_dim),
                           d["a"], d["b"], params["conv1d.weight"], params["A_log"], params["dt_bias"],
                           params["norm.weight"], dtype, d.get("conv_state"), d.get("rec_state"), chunk=chunk,
                           checkpoint_offsets=offsets)


def check(shape, dtype, ours, ref, offsets=(), what=""):
    out, cs, rs, st_ck, cv_ck = ours
    r_out, r_cs, r_rs, r_cv, r_st = ref
    if dtype == "bf16":
        assert_bf16_close(out, r_out, what + " out")
    else:
        assert_f32_close(out, r_out, 5e-5, what + " out")
    assert_bit_exact(cs, r_cs, what + " conv state")
    assert_state_close(rs, r_rs, what + " state")
    for i, off in enumerate(offsets):
        assert_bit_exact(cv_ck[i], r_cv[off], f"{what} conv checkpoint {off}")
        assert_state_close(st_ck[i], r_st[off], f"{what} state checkpoint {off}")


@pytest.mark.parametrize("register_kernel", [False, True])
@pytest.mark.parametrize("dtype", ["bf16", "f32"])
@pytest.mark.parametrize("T,offsets", [(1, (1,)), (4, (1, 2, 4)), (8, (3, 8))])
def test_token_by_token_small(dtype, T, offsets, register_kernel):
    shape = W.SHAPE_TINY
    m, params = make_layer(shape, dtype)
    d = mixer_inputs(shape, 3, T, dtype, seed=10 + T, with_state=True)
    check(shape, dtype, run_ours(m, shape, d, dtype, True, offsets, register_kernel),
          run_oracle(shape, params, d, dtype, chunk=False, offsets=offsets), offsets, f"tbt T{T}")


@pytest.mark.parametrize("d_head,T", [(64, 1), (64, 5), (128, 3)])
def test_token_by_token_head_dims(d_head, T):
    shape = W.LayerShape(256, 2, 4, d_head, d_head)
    m, params = make_layer(shape, "bf16")
    d = mixer_inputs(shape, 5, T, "bf16", seed=31 + T, with_state=True)
    offs = tuple(range(1, T + 1))
    check(shape, "bf16", run_ours(m, shape, d, "bf16", True, offs),
          run_oracle(shape, params, d, "bf16", chunk=False, offsets=offs), offs, f"tbt d{d_head}")


def test_token_by_token_unaligned_strides_fall_back():
    """Projection outputs with a token stride that is not a multiple of 16
    bytes cannot be bulk-copied; the register-tile kernel takes over."""
    from visionstack_b200 import _lib
    shape = W.SHAPE_TINY
    m, params = make_layer(shape, "bf16")
    d = mixer_inputs(shape, 2, 2, "bf16", seed=77, with_state=True)
    dev = torch.device("cuda")
    t = lambda a: torch.from_numpy(a).to(dev).to(torch.bfloat16)  # noqa: E731
    wide = torch.zeros(2, 2, shape.conv_dim + 3, dtype=torch.bfloat16, device=dev)
    wide[..., :shape.conv_dim] = t(d["mixed"])
    mixed = wide[..., :shape.conv_dim]
    assert mixed.stride(1) % 8 != 0
    out = m.mixer(mixed, t(d["z"]), t(d["b"]), t(d["a"]), conv_state=t(d["conv_state"]),
                  rec_state=torch.from_numpy(d["rec_state"]).to(dev), token_by_token=True)
    torch.cuda.synchronize()
    ref = run_oracle(shape, params, d, "bf16", chunk=False)
    assert_bf16_close(out, ref[0], "unaligned")
    assert _lib.device_error() == 0


def test_token_by_token_without_state():
    shape = W.SHAPE_TINY
    m, params = make_layer(shape, "bf16")
    d = mixer_inputs(shape, 2, 3, "bf16", seed=5, with_state=False)
    check(shape, "bf16", run_ours(m, shape, d, "bf16", True), run_oracle(shape, params, d, "bf16", chunk=False))


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
@pytest.mark.parametrize("T,with_state,offsets", [
    (3, False, (1, 3)), (64, True, (64,)), (200, True, (1, 17, 64, 100, 128, 199, 200)), (130, False, ())])
def test_chunked_small(dtype, T, with_state, offsets):
    shape = W.SHAPE_TINY
    m, params = make_layer(shape, dtype)
    d = mixer_inputs(shape, 2, T, dtype, seed=20 + T, with_state=with_state)
    check(shape, dtype, run_ours(m, shape, d, dtype, False, offsets),
          run_oracle(shape, params, d, dtype, chunk=True, offsets=offsets), offsets, f"chunk T{T}")


@pytest.mark.parametrize("d_head", [64, 128])
def test_chunked_head_dims(d_head):
    shape = W.LayerShape(256, 2, 4, d_head, d_head)
    m, params = make_layer(shape, "bf16")
    d = mixer_inputs(shape, 1, 150, "bf16", seed=3, with_state=True)
    check(shape, "bf16", run_ours(m, shape, d, "bf16", False, (70, 150)),
          run_oracle(shape, params, d, "bf16", chunk=True, offsets=(70, 150)), (70, 150), f"d{d_head}")


@pytest.mark.parametrize("register_kernel", [False, True])
def test_decode_step_qwen_shape(register_kernel):
    """One decode step at the decode benchmark's shape (B64, 16/32 heads, d128)."""
    from visionstack_b200 import _lib
    shape = W.SHAPE_QWEN
    m, params = make_layer(shape, "bf16")
    d = mixer_inputs(shape, 64, 1, "bf16", seed=2, with_state=True)
    check(shape, "bf16", run_ours(m, shape, d, "bf16", True, register_kernel=register_kernel),
          run_oracle(shape, params, d, "bf16", chunk=False), what="decode B64")
    assert _lib.device_error() == 0


def test_prefill_qwen_shape():
    """Chunked prefill at the prefill benchmark's head layout (B1, T320)."""
    shape = W.SHAPE_QWEN
    m, params = make_layer(shape, "bf16")
    d = mixer_inputs(shape, 1, 320, "bf16", seed=3, with_state=False)
    check(shape, "bf16", run_ours(m, shape, d, "bf16", False, (100, 256, 320)),
          run_oracle(shape, params, d, "bf16", chunk=True, offsets=(100, 256, 320)), (100, 256, 320), "prefill")


def test_inplace_state_update_matches_out_of_place():
    shape = W.SHAPE_QWEN
    m, _ = make_layer(shape, "bf16")
    d = mixer_inputs(shape, 8, 1, "bf16", seed=9, with_state=True)
    dev = torch.device("cuda")
    t = lambda a: torch.from_numpy(a).to(dev).to(torch.bfloat16)  # noqa: E731
    S = torch.from_numpy(d["rec_state"]).to(dev)
    S_copy = S.clone()
    out_a = m.mixer(t(d["mixed"]), t(d["z"]), t(d["b"]), t(d["a"]), conv_state=t(d["conv_state"]), rec_state=S,
                    rec_state_out=S, token_by_token=True)
    S_b = torch.empty_like(S)
    out_b = m.mixer(t(d["mixed"]), t(d["z"]), t(d["b"]), t(d["a"]), conv_state=t(d["conv_state"]),
                    rec_state=S_copy, rec_state_out=S_b, token_by_token=True)
    torch.cuda.synchronize()
    assert torch.equal(out_a, out_b) and torch.equal(S, S_b)


def test_chunked_equals_token_by_token_at_scale():
    """Size-independent property at the decode batch: 64 tokens through the
    chunked kernel == 64 single-token decode launches, from the same state."""
    shape = W.SHAPE_QWEN
    m, _ = make_layer(shape, "bf16")
    B, T = 64, 64
    d = mixer_inputs(shape, B, T, "bf16", seed=4, with_state=True)
    dev = torch.device("cuda")
    t = lambda a: torch.from_numpy(a).to(dev).to(torch.bfloat16)  # noqa: E731
    mixed, z, b, a = t(d["mixed"]), t(d["z"]), t(d["b"]), t(d["a"])
    cs0, S0 = t(d["conv_state"]), torch.from_numpy(d["rec_state"]).to(dev)
    S_chunk = torch.empty_like(S0)
    cs_chunk = torch.empty_like(cs0)
    out_chunk = m.mixer(mixed, z, b, a, conv_state=cs0, rec_state=S0, conv_state_out=cs_chunk,
                        rec_state_out=S_chunk, token_by_token=False)
    S = S0.clone()
    cs = cs0.clone()
    outs = []
    for i in range(T):
        cs_next = torch.empty_like(cs)
        outs.append(m.mixer(mixed[:, i:i + 1], z[:, i:i + 1], b[:, i:i + 1], a[:, i:i + 1], conv_state=cs,
                            rec_state=S, conv_state_out=cs_next, rec_state_out=S, token_by_token=True))
        cs = cs_next
    torch.cuda.synchronize()
    # two implementations, each within tolerance of the reference
    assert_bf16_close(torch.cat(outs, 1), out_chunk, "chunk vs decode out", scale=2.0)
    assert_state_close(S, S_chunk, "chunk vs decode state", scale=2.0)
    assert torch.equal(cs, cs_chunk)


def test_mixer_plan_matches_mixer():
    """The prepared-call API launches the same kernel with pre-bound weights."""
    shape = W.SHAPE_QWEN
    m, _ = make_layer(shape, "bf16")
    d = mixer_inputs(shape, 16, 1, "bf16", seed=12, with_state=True)
    dev = torch.device("cuda")
    t = lambda a: torch.from_numpy(a).to(dev).to(torch.bfloat16)  # noqa: E731
    args = (t(d["mixed"]), t(d["z"]), t(d["b"]), t(d["a"]))
    S1 = torch.from_numpy(d["rec_state"]).to(dev)
    S2 = S1.clone()
    cs1, cs2 = torch.empty(16, shape.conv_dim, 3, dtype=torch.bfloat16, device=dev), \
        torch.empty(16, shape.conv_dim, 3, dtype=torch.bfloat16, device=dev)
    o1 = m.mixer(*args, conv_state=t(d["conv_state"]), rec_state=S1, conv_state_out=cs1, rec_state_out=S1)
    plan = m.mixer_plan(16, 1, torch.bfloat16, dev)
    o2 = torch.empty_like(o1)
    plan(*args, t(d["conv_state"]), S2, cs2, S2, o2)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(S1, S2) and torch.equal(cs1, cs2)


PREFILL_FORMS = {"default": {}, "prep_in_kernel": {"prep_in_kernel_prefill": True}, "single_kernel": {"fused_prefill": True}}


@pytest.mark.parametrize("form", list(PREFILL_FORMS))
@pytest.mark.parametrize("B,T,with_state,offsets", [
    (2, 200, True, (1, 37, 64, 100, 128, 199, 200)),
    (1, 64, False, (64,)),
    (3, 7, True, (3, 7)),
    (1, 513, False, (256, 500, 513)),
    (2, 130, True, (65, 66, 67, 129)),
])
def test_tensor_core_prefill_vs_oracle(B, T, with_state, offsets, form):
    """The tcgen05 chunked kernels (bf16, head dim 128) against the oracle, with
    sub-chunk and chunk-boundary checkpoints, ragged last chunks and T < 64:
    the default two-kernel form (parallel preparation pass through a
    workspace, then the sequential pass), the single kernel whose producer
    warps prepare each chunk two chunks ahead of the state pass, and the older
    single kernel that prepares each chunk on the state's critical path."""
    from visionstack_b200 import _lib
    shape = W.LayerShape(256, 2, 4, 128, 128)
    m, params = make_layer(shape, "bf16")
    d = mixer_inputs(shape, B, T, "bf16", seed=40 + T, with_state=with_state)
    check(shape, "bf16", run_ours(m, shape, d, "bf16", False, offsets, **PREFILL_FORMS[form]),
          run_oracle(shape, params, d, "bf16", chunk=True, offsets=offsets), offsets, f"tc T{T} {form}")
    assert _lib.device_error() == 0


@pytest.mark.parametrize("form", ["default", "prep_in_kernel"])
def test_prefill_chains_split_across_ctas(form):
    """More (batch, value head) chains than SMs: the sequential kernel runs one CTA per SM,
    cuts the chains' chunks into equal runs and hands the state from one CTA to the next
    (chain heads, tails and whole chains; checkpoints on both sides of a hand-off)."""
    from visionstack_b200 import _lib
    shape = W.LayerShape(256, 2, 4, 128, 128)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    B, T = sms // shape.num_v_heads + 3, 200  # B * 4 chains > SMs; 4 chunks per chain
    offs = (1, 37, 64, 100, 128, 199, 200)
    m, params = make_layer(shape, "bf16")
    d = mixer_inputs(shape, B, T, "bf16", seed=77, with_state=True)
    check(shape, "bf16", run_ours(m, shape, d, "bf16", False, offs, **PREFILL_FORMS[form]),
          run_oracle(shape, params, d, "bf16", chunk=True, offsets=offs), offs, f"split chains {form}")
    assert _lib.device_error() == 0


@pytest.mark.parametrize("form", ["default", "prep_in_kernel"])
@pytest.mark.parametrize("rep", [1, 4])
def test_prefill_gqa_groupings(rep, form):
    """Key heads shared by 1 or 4 value heads (the preparation pass handles
    every value head of a key head in one CTA)."""
    from visionstack_b200 import _lib
    shape = W.LayerShape(256, 2, 2 * rep, 128, 128)
    m, params = make_layer(shape, "bf16")
    d = mixer_inputs(shape, 2, 150, "bf16", seed=60 + rep, with_state=True)
    offs = (10, 64, 150)
    check(shape, "bf16", run_ours(m, shape, d, "bf16", False, offs, **PREFILL_FORMS[form]),
          run_oracle(shape, params, d, "bf16", chunk=True, offsets=offs), offs, f"rep{rep} {form}")
    assert _lib.device_error() == 0


def test_tensor_core_prefill_matches_cuda_core_kernel():
    shape = W.SHAPE_QWEN
    m, _ = make_layer(shape, "bf16")
    d = mixer_inputs(shape, 2, 300, "bf16", seed=8, with_state=True)
    dev = torch.device("cuda")
    t = lambda a: torch.from_numpy(a).to(dev).to(torch.bfloat16)  # noqa: E731
    S0 = torch.from_numpy(d["rec_state"]).to(dev)
    outs = []
    for kw in ({}, {"fused_prefill": True}, {"cuda_core_prefill": True}, {"prep_in_kernel_prefill": True}):
        S = torch.empty_like(S0)
        o = m.mixer(t(d["mixed"]), t(d["z"]), t(d["b"]), t(d["a"]), conv_state=t(d["conv_state"]), rec_state=S0,
                    rec_state_out=S, token_by_token=False, **kw)
        outs.append((o, S))
    torch.cuda.synchronize()
    for i, name in ((1, "single-kernel"), (2, "cuda-core"), (3, "prep-in-kernel")):
        assert_bf16_close(outs[0][0], outs[i][0], f"default vs {name} out", scale=2.0)
        assert_state_close(outs[0][1], outs[i][1], f"default vs {name} state", scale=2.0)


def test_prefill_plan_matches_mixer():
    """The prepared-call API on the chunked path (workspace kept by the plan)."""
    shape = W.SHAPE_QWEN
    m, _ = make_layer(shape, "bf16")
    B, T = 2, 200
    d = mixer_inputs(shape, B, T, "bf16", seed=13, with_state=True)
    dev = torch.device("cuda")
    t = lambda a: torch.from_numpy(a).to(dev).to(torch.bfloat16)  # noqa: E731
    args = (t(d["mixed"]), t(d["z"]), t(d["b"]), t(d["a"]))
    S0 = torch.from_numpy(d["rec_state"]).to(dev)
    S1, S2 = torch.empty_like(S0), torch.empty_like(S0)
    cs1 = torch.empty(B, shape.conv_dim, 3, dtype=torch.bfloat16, device=dev)
    cs2 = torch.empty_like(cs1)
    o1 = m.mixer(*args, conv_state=t(d["conv_state"]), rec_state=S0, conv_state_out=cs1, rec_state_out=S1,
                 token_by_token=False)
    plan = m.mixer_plan(B, T, torch.bfloat16, dev, token_by_token=False)
    o2 = torch.empty_like(o1)
    for _ in range(2):
        plan(*args, t(d["conv_state"]), S0, cs2, S2, o2)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(S1, S2) and torch.equal(cs1, cs2)
