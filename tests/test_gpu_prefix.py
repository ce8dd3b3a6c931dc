"""Prefix-state snapshots through pinned host memory on the copy stream.

* A prompt is prefilled with checkpoints at 32 and 64; its snapshot is
  spliced back at 64 for a second prompt that shares 72 tokens.  The restored
  states equal the recorded checkpoints bit for bit, and continuing from them
  reproduces the unsplit pass (ShadowBoxer/core/caches.py:301-340 splice,
  the trajectory property of gate3_models.py:1247-1276).
* A snapshot is taken while the layer keeps decoding on the same cache: the
  snapshot holds the states of the moment it was taken, and the layer no
  longer updates the snapshotted state tensor in place.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.helpers import max_abs
from tests.test_gpu_mixer import make_layer
from visionstack_b200 import PrefixStateCache, Qwen3_5HybridCache, snapshot_prefix_state
from visionstack_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _hidden(shape, B, T, seed):
    x = np.random.default_rng(seed).standard_normal((B, T, shape.hidden_size)).astype(np.float32)
    return torch.from_numpy(x).cuda().to(torch.bfloat16)


def test_snapshot_splice_matches_unsplit_pass():
    shape = W.SHAPE_TINY
    m, _ = make_layer(shape, "bf16", seed=11)
    B, T = 2, 96
    x = _hidden(shape, B, T, 4)
    toks = list(range(1000, 1000 + T))
    with torch.inference_mode():
        c = Qwen3_5HybridCache(record_checkpoints=True, checkpoint_positions=[32, 64])
        c.resolve_active_checkpoints(0, T)
        full = m(x, cache=c)
        c.past_seen_tokens = T
        ref_conv64 = c.conv_checkpoints[64][0].clone()
        ref_rec64 = c.recurrent_checkpoints[64][0].clone()
        pc = PrefixStateCache()
        st = pc.insert_prefix_state(toks, x, c)
        assert st is not None and st.available_offsets == (32, 64, 96)
        st.synchronize()
        assert st.is_ready()
        # a prompt sharing 72 tokens splices at the largest offset <= 72
        prompt = toks[:72] + [7] * 30
        got = pc.lookup_prefix_splice(prompt, torch.device("cuda"))
        assert got is not None
        rc, hidden, off = got
        assert off == 64 and rc.past_seen_tokens == 64 and pc.splice_hits == 1
        assert torch.equal(rc.conv_states[0], ref_conv64)
        assert torch.equal(rc.recurrent_states[0], ref_rec64)
        assert torch.equal(hidden, x[:, :64])
        tail = m(x[:, 64:], cache=rc)
    spliced = torch.cat([full[:, :64], tail], 1)
    assert max_abs(full, spliced) <= 0.0625 and float((full - spliced).abs().float().mean()) < 2e-3


def test_snapshot_is_not_overwritten_by_later_steps():
    shape = W.SHAPE_TINY
    m, _ = make_layer(shape, "bf16", seed=12)
    B = 3
    with torch.inference_mode():
        c = Qwen3_5HybridCache()
        m(_hidden(shape, B, 40, 5), cache=c)
        c.past_seen_tokens = 40
        owned = c.recurrent_states[0]
        m(_hidden(shape, B, 1, 6), cache=c)  # our own state: updated in place
        assert c.recurrent_states[0] is owned
        before_rec = owned.clone()
        before_conv = c.conv_states[0].clone()
        st = snapshot_prefix_state(list(range(41)), None, c)
        for i in range(8):  # keep decoding at once, without waiting for the copies
            m(_hidden(shape, B, 1, 7 + i), cache=c)
        assert c.recurrent_states[0] is not owned
        st.synchronize()
        assert torch.equal(st.recurrent_states[0], before_rec.cpu())
        assert torch.equal(st.conv_states[0], before_conv.cpu())
        assert st.recurrent_states[0].is_pinned()
        rc, _, off = st.restore(torch.device("cuda"))
        assert off == 41 and torch.equal(rc.recurrent_states[0], before_rec)
        # a restored state belongs to the new cache: the next step updates it in place
        mine = rc.recurrent_states[0]
        m(_hidden(shape, B, 1, 20), cache=rc)
        assert rc.recurrent_states[0] is mine
