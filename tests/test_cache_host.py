"""Host logic of the hybrid cache against the reference's recorded behaviour
(tests/golden/cache.json) and its rollback rules (cache.py:131-244)."""
from __future__ import annotations

import json
import os

import pytest
import torch

from visionstack_b200 import Qwen3_5HybridCache
from visionstack_b200.cache import is_owned, mark_owned

GOLD = os.path.join(os.path.dirname(__file__), "golden", "cache.json")


def fixture():
    with open(GOLD) as f:
        return json.load(f)


@pytest.mark.parametrize("case", fixture()["resolve"])
def test_resolve_active_checkpoints(case):
    c = Qwen3_5HybridCache(record_checkpoints=True, checkpoint_positions=case["requested"],
                           min_checkpoint_token=case["min_tok"], structural_checkpoints=case["structural"])
    assert c.resolve_active_checkpoints(case["past"], case["T"]) == case["result"]


@pytest.mark.parametrize("case", fixture()["structural"])
def test_derive_structural_checkpoints(case):
    ms, cps = Qwen3_5HybridCache.derive_structural_checkpoints(case["tokens"])
    assert ms == case["min_snap"] and cps == case["cps"]


def test_reference_gate_anchor_assertions():
    # gate2_caches.py:55-70: the vision_end anchor and the 0.82 snapped position
    toks = [248045, 872, 198, 248053] + [248056] * 16 + [248054] + list(range(200, 260)) + [248044]
    ms, cps = Qwen3_5HybridCache.derive_structural_checkpoints(toks)
    assert ms == 21 and 21 in cps and len(cps) >= 3
    c = Qwen3_5HybridCache(record_checkpoints=True, min_checkpoint_token=4, structural_checkpoints=cps)
    auto = c.resolve_active_checkpoints(0, 53)
    assert 44 in auto and 21 in auto


def _filled(B=3):
    c = Qwen3_5HybridCache(record_checkpoints=True, checkpoint_positions=[12, 16])
    c.past_seen_tokens = 20
    c.rope_deltas = torch.tensor([[-4]] * B)
    c.conv_states[0] = torch.randn(B, 16, 3).to(torch.bfloat16)
    c.recurrent_states[0] = torch.randn(B, 2, 8, 8)
    for p in (12, 16):
        c.conv_checkpoints[p] = {0: torch.randn(B, 16, 3).to(torch.bfloat16)}
        c.recurrent_checkpoints[p] = {0: torch.randn(B, 2, 8, 8)}
    c.key_cache[3] = torch.randn(B, 2, 20, 4)
    c.value_cache[3] = torch.randn(B, 2, 20, 4)
    return c


def test_select_batch_item_rolls_back_to_checkpoint():
    c = _filled()
    s = c.select_batch_item(1, total_valid_tokens=16)
    assert s.past_seen_tokens == 16
    assert torch.equal(s.recurrent_states[0], c.recurrent_checkpoints[16][0][1:2])
    assert torch.equal(s.conv_states[0], c.conv_checkpoints[16][0][1:2])
    assert s.key_cache[3].shape == (1, 2, 16, 4)
    assert s.recurrent_states[0].dtype == torch.float32


def test_select_batch_item_without_checkpoint_keeps_current_states():
    # no checkpoint at 18: the reference falls back to the current states (cache.py:212-227)
    c = _filled()
    s = c.select_batch_item(2, total_valid_tokens=18)
    assert torch.equal(s.recurrent_states[0], c.recurrent_states[0][2:3])
    assert s.key_cache[3].shape[2] == 18


def test_extract_checkpoint_and_errors():
    c = _filled()
    e = c.extract_checkpoint(12)
    assert e.past_seen_tokens == 12 and torch.equal(e.recurrent_states[0], c.recurrent_checkpoints[12][0])
    assert e.recurrent_states[0].data_ptr() != c.recurrent_checkpoints[12][0].data_ptr()
    with pytest.raises(KeyError):
        c.extract_checkpoint(13)
    same = c.extract_checkpoint(20)  # == past_seen_tokens: a plain clone
    assert torch.equal(same.recurrent_states[0], c.recurrent_states[0])


def test_clone_and_expand_repeats_rows():
    c = _filled(B=1)
    e = c.clone_and_expand(4, record_checkpoints=True, checkpoint_positions=[21, 22])
    assert e.recurrent_states[0].shape[0] == 4 and e.rope_deltas.shape == (4, 1)
    assert torch.equal(e.recurrent_states[0][3], c.recurrent_states[0][0])
    assert e.record_checkpoints and e.resolve_active_checkpoints(20, 2) == [21, 22]


def test_ownership_tags_do_not_survive_clones():
    c = _filled()
    t = mark_owned(torch.zeros(2), c, 0)
    assert is_owned(t, c, 0) and not is_owned(t, c, 1)
    e = c.clone_and_expand(1)
    assert not is_owned(t, e, 0)
    assert not is_owned(t.clone(), c, 0)
