"""Host logic of the prefix-state cache (ShadowBoxer/core/caches.py:58-340):
offset selection, best-offset resolution, splice lookup and LRU order.  The
snapshots here are built by hand from host tensors; copies need a GPU and are
covered by tests/test_gpu_prefix.py."""
from __future__ import annotations

import pytest
import torch

from visionstack_b200 import Qwen3_5HybridCache
from visionstack_b200.prefix import (PinnedPrefixState, PrefixStateCache, common_prefix_len, snapshot_offsets,
                                     snapshot_prefix_state)


def test_common_prefix_len():
    assert common_prefix_len([1, 2, 3], [1, 2, 4]) == 2
    assert common_prefix_len([], [1]) == 0
    assert common_prefix_len([5, 6], [5, 6, 7]) == 2


def test_snapshot_offsets_rules():
    conv = {8: {0: 1}, 16: {0: 1}, 40: {0: 1}, 0: {0: 1}}
    rec = {8: {0: 1}, 24: {0: 1}, 40: {0: 1}}
    # both kinds recorded, 1 <= cp <= full_len, plus full_len when current states exist
    assert snapshot_offsets(conv, rec, 32, True) == (8, 32)
    assert snapshot_offsets(conv, rec, 48, False) == (8, 40)
    assert snapshot_offsets({}, {}, 10, False) == ()


def _state(tokens, offsets, sig=()):
    return PinnedPrefixState(prefix_tokens=tuple(tokens), vision_signature=tuple(sig), prefix_hidden=None,
                             conv_states={}, recurrent_states={}, key_cache={}, value_cache={}, rope_deltas=None,
                             available_offsets=tuple(offsets))


def test_resolve_best_offset():
    st = _state(range(40), (8, 24, 40))
    assert st.resolve_best_offset(30) == 24
    assert st.resolve_best_offset(7) is None
    assert st.resolve_best_offset(100) == 40
    assert _state(range(12), ()).resolve_best_offset(12) == 12


def test_find_prefers_longest_then_recent_and_never_whole_prompt():
    c = PrefixStateCache(max_prefix_entries=2)
    a = _state(range(64), (16, 32, 64))
    b = _state(list(range(20)) + [999] * 44, (16, 20, 64))
    c._prefix_cache[a.prefix_tokens] = a
    c._prefix_cache[b.prefix_tokens] = b
    hit = c.find(list(range(70)))
    assert hit is not None and hit[1] is a and hit[2] == 64
    # the whole prompt is never spliced: at most total_len - 1
    hit = c.find(list(range(64)))
    assert hit[1] is a and hit[2] == 32
    # a prompt that diverges at 25: b reaches 20, a 16
    hit = c.find(list(range(25)) + [7] * 10)
    assert hit[1] is b and hit[2] == 20
    assert c.find(list(range(15))) is None  # under 16 tokens
    assert c.find(list(range(40)), vision_signature=("img",)) is None


def test_lru_eviction_and_keys():
    c = PrefixStateCache(max_prefix_entries=2)
    for i in range(3):
        st = _state([i] * 20, (20,), sig=("v",) if i == 2 else ())
        key = (st.prefix_tokens, st.vision_signature) if st.vision_signature else st.prefix_tokens
        c._prefix_cache[key] = st
        while len(c._prefix_cache) > c.max_prefix_entries:
            c._prefix_cache.popitem(last=False)
    assert len(c) == 2 and tuple([0] * 20) not in c._prefix_cache


def test_snapshot_requires_cuda_tensors():
    cache = Qwen3_5HybridCache()
    cache.conv_states[0] = torch.zeros(1, 8, 3)
    cache.recurrent_states[0] = torch.zeros(1, 2, 4, 4)
    with pytest.raises(RuntimeError):
        snapshot_prefix_state(list(range(20)), None, cache)
    assert snapshot_prefix_state([], None, cache) is None
