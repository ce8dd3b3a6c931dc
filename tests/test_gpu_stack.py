"""The hybrid decoder stack (three Gated DeltaNet layers on the CUDA token mixer, one gated
attention layer, MLPs, norms) against the reference's own text stack run on the host
(``tests/golden/make_stack_golden.py``): the same seeded parameters and calls - a 70-token prefill
into a hybrid cache, three decode steps, a 4-token step, and a cache-less call under a 2-D mask.

Tolerances, max abs over hidden states of magnitude up to ~4.4: fp32 2e-3 (GEMMs of cuBLAS vs
the host, the mixer's fp32 path); bf16 0.125 with a mean abs below 0.01 (one bf16 ulp at 4 is
0.03; roundings of different GEMM orders propagate through four layers).
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from visionstack_b200 import Qwen3_5HybridCache, Qwen3_5TextConfig
from visionstack_b200 import workloads as W
from visionstack_b200.stack import Qwen3_5TextModel, StackDecodeGraph

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
TDT = {"f32": torch.float32, "bf16": torch.bfloat16}
TOL = {"f32": (2e-3, 2e-4), "bf16": (0.125, 0.01)}


def build(dtype: str):
    model = Qwen3_5TextModel(Qwen3_5TextConfig(**W.STACK_TINY)).eval().to(TDT[dtype])
    shapes = {k: tuple(v.shape) for k, v in model.state_dict().items()}
    params = W.make_stack_params(shapes, seed=7, dtype=dtype)
    model.load_state_dict({k: torch.from_numpy(v).to(TDT[dtype]) for k, v in params.items()}, strict=True)
    for mod in model.modules():  # float32 after the load, as the fixture's script does
        for k in ("A_log", "dt_bias"):
            if hasattr(mod, k):
                getattr(mod, k).data = getattr(mod, k).data.float()
    return model.cuda()


def close(ours: torch.Tensor, ref: np.ndarray, dtype: str, what: str):
    o = ours.float().cpu().numpy()
    assert o.shape == ref.shape, what
    d = np.abs(o - ref)
    mx, mean = TOL[dtype]
    assert np.isfinite(o).all(), what
    assert d.max() <= mx and d.mean() <= mean, f"{what}: max {d.max():.3e} mean {d.mean():.3e}"


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("kv_capacity", [0, 96])
def test_stack_matches_reference(dtype, kv_capacity):
    ref = np.load(GOLDEN / f"stack_tiny_{dtype}.npz")
    model = build(dtype)
    ids, spans, mask = W.make_stack_calls(W.STACK_TINY)
    ids_t = torch.from_numpy(ids).cuda()
    with torch.inference_mode():
        cache = Qwen3_5HybridCache()
        cache.kv_capacity = kv_capacity
        for i, (a, b) in enumerate(spans):
            o = model(input_ids=ids_t[:, a:b], past_key_values=cache, use_cache=True)
            close(o.last_hidden_state, ref[f"h{i}"], dtype, f"call {i} tokens {a}..{b}")
        assert cache.past_seen_tokens == 77
        close(cache.key_cache[3], ref["key3"], dtype, "key cache of the attention layer")
        close(cache.conv_states[0], ref["conv0"], dtype, "conv state of layer 0")
        S, Sr = cache.recurrent_states[0].float().cpu().numpy(), ref["rec0"]
        assert np.abs(S - Sr).max() <= 2e-3 * np.abs(Sr).max() * (1 if dtype == "f32" else 20), "state of layer 0"
        o = model(input_ids=ids_t[:, :40], attention_mask=torch.from_numpy(mask).cuda())
        close(o.last_hidden_state, ref["h_mask"], dtype, "masked call")


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_decode_graph_matches_eager_decode(dtype):
    """Decode steps replayed from one CUDA graph (static KV buffers, positions on the device, conv
    state copied back) against the eager decode path, after the same prefill."""
    model = build(dtype)
    ids, _, _ = W.make_stack_calls(W.STACK_TINY)
    ids_t = torch.from_numpy(ids).cuda()
    P, N = 70, ids.shape[1]
    tol = {"f32": (1e-4, 1e-5), "bf16": (0.07, 0.004)}[dtype]
    with torch.inference_mode():
        caches = []
        for _ in range(2):
            c = Qwen3_5HybridCache()
            c.kv_capacity = 96
            model(input_ids=ids_t[:, :P], past_key_values=c, use_cache=True)
            caches.append(c)
        ce, cg = caches
        dg = StackDecodeGraph(model, cg, ids_t)
        for p in range(P, N):
            he = model(input_ids=ids_t[:, p:p + 1], past_key_values=ce, use_cache=True).last_hidden_state
            hg = dg.step().clone()
            d = (he.float() - hg.float()).abs()
            assert d.max() <= tol[0] and d.mean() <= tol[1], f"step {p}: max {d.max():.3e} mean {d.mean():.3e}"
        dg.finish()
        torch.cuda.synchronize()
    assert cg.past_seen_tokens == ce.past_seen_tokens == N
    for l in (0, 1, 2):
        assert torch.equal(cg.conv_states[l], ce.conv_states[l]) or dtype == "bf16"
        d = (cg.recurrent_states[l] - ce.recurrent_states[l]).abs().max().item()
        assert d <= 1e-3 * ce.recurrent_states[l].abs().max().item() * (1 if dtype == "f32" else 20)
    assert cg.key_cache[3].shape == ce.key_cache[3].shape
    assert (cg.key_cache[3].float() - ce.key_cache[3].float()).abs().max().item() <= tol[0]
