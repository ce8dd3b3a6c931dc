"""Prefix-cache snapshots of the hybrid cache in pinned host memory.

The reference keeps, per shared prompt prefix, a pinned-host copy of every
layer's conv / recurrent state, its recorded checkpoints, the attention KV
cache sliced to the longest usable offset, the prefix hidden states and the
rope deltas (ShadowBoxer/core/caches.py:58-128 ``PinnedPrefixState``,
:203-299 ``PromptEmbedCache.insert_prefix_state``), and splices the longest
usable snapshot back into a new cache for a later prompt
(:301-340 ``lookup_prefix_splice``).  The reference copies synchronously
(core/env.py:143-157 ``_pin_cpu_tensor``: ``copy_(non_blocking=False)``).

Here the same records, offsets and restore rules run asynchronously:

* ``snapshot`` enqueues the device-to-host copies on a dedicated copy
  stream, ordered after the producing stream by an event, into one pinned
  arena per snapshot (a single allocation, every tensor a 256-byte aligned
  view).  The host returns at once; ``PinnedPrefixState.ready`` marks the
  copies' completion.  The snapshotted device tensors stay alive through the
  caching allocator (``record_stream``) until the copies finish, and their
  in-place ownership tag is cleared, so the next layer step writes fresh
  tensors instead of the ones still being copied.
* ``restore`` copies host-to-device on the same copy stream into new device
  tensors and makes the caller's stream wait for them; the restored
  recurrent states belong to the new cache (the layer may update them in
  place).

Snapshots and restores need CUDA tensors: there is no host-only path.
"""
from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Sequence, Tuple

import torch

from .cache import Qwen3_5HybridCache, _OWNER_ATTR, mark_owned

_ALIGN = 256


def common_prefix_len(a: Sequence[int], b: Sequence[int]) -> int:
    """Length of the longest common prefix of two token sequences (the
    reference calls ``MOSSImageTokenizer.find_common_prefix`` for this)."""
    n = min(len(a), len(b))
    i = 0
    while i < n and int(a[i]) == int(b[i]):
        i += 1
    return i


def snapshot_offsets(conv_checkpoints: Dict[int, Dict[int, Any]], recurrent_checkpoints: Dict[int, Dict[int, Any]],
                     full_len: int, have_current: bool) -> Tuple[int, ...]:
    """Offsets a snapshot can restore to (caches.py:223-259): checkpoints
    1 <= cp <= full_len recorded for both state kinds, plus full_len itself
    when the cache holds current states."""
    conv_ok = {int(cp) for cp, m in conv_checkpoints.items() if 1 <= int(cp) <= full_len and m}
    rec_ok = {int(cp) for cp, m in recurrent_checkpoints.items() if 1 <= int(cp) <= full_len and m}
    offs = conv_ok & rec_ok
    if have_current:
        offs.add(int(full_len))
    return tuple(sorted(offs))


_COPY_STREAMS: Dict[int, torch.cuda.Stream] = {}


def copy_stream(device: torch.device) -> torch.cuda.Stream:
    """The per-device stream that carries snapshot and restore copies."""
    dev = torch.device(device)
    if dev.type != "cuda":
        raise RuntimeError("prefix snapshots need CUDA tensors")
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    s = _COPY_STREAMS.get(idx)
    if s is None:
        s = torch.cuda.Stream(device=idx)
        _COPY_STREAMS[idx] = s
    return s


class _PinnedArena:
    """One pinned host allocation carved into 256-byte aligned views shaped like `like`."""

    def __init__(self, like: Sequence[torch.Tensor]):
        offs, total = [], 0
        for t in like:
            offs.append(total)
            total += (t.numel() * t.element_size() + _ALIGN - 1) // _ALIGN * _ALIGN
        self.nbytes = total
        self.buf = torch.empty(max(total, _ALIGN), dtype=torch.uint8, pin_memory=True)
        self.views: List[torch.Tensor] = []
        for t, o in zip(like, offs):
            n = t.numel() * t.element_size()
            if n == 0:
                self.views.append(torch.empty(t.shape, dtype=t.dtype))
            else:
                self.views.append(self.buf[o:o + n].view(t.dtype).view(t.shape))


def _release_ownership(t: torch.Tensor) -> None:
    if getattr(t, _OWNER_ATTR, None) is not None:
        setattr(t, _OWNER_ATTR, None)


def _d2h(srcs: List[torch.Tensor]) -> Tuple[_PinnedArena, torch.cuda.Event]:
    """Enqueue pinned copies of `srcs` on the copy stream after the current
    stream's work; returns the arena and the copies' completion event."""
    dev = srcs[0].device
    cs = copy_stream(dev)
    produced = torch.cuda.Event()
    produced.record(torch.cuda.current_stream(dev))
    arena = _PinnedArena(srcs)
    with torch.cuda.stream(cs):
        cs.wait_event(produced)
        for s, v in zip(srcs, arena.views):
            v.copy_(s, non_blocking=True)
            s.record_stream(cs)
    done = torch.cuda.Event()
    done.record(cs)
    return arena, done


def _h2d(host: List[torch.Tensor], device: torch.device, after: Optional[torch.cuda.Event]) -> List[torch.Tensor]:
    """Device copies of pinned `host` tensors, made on the copy stream once
    `after` (the snapshot's completion) has passed; the caller's stream waits
    for them."""
    dev = torch.device(device)
    cur = torch.cuda.current_stream(dev)
    cs = copy_stream(dev)
    outs = [torch.empty(h.shape, dtype=h.dtype, device=dev) for h in host]
    cs.wait_stream(cur)  # the new tensors' memory is free in the current stream's order
    with torch.cuda.stream(cs):
        if after is not None:
            cs.wait_event(after)
        for h, o in zip(host, outs):
            o.copy_(h, non_blocking=True)
            o.record_stream(cs)
    cur.wait_stream(cs)
    return outs


@dataclass
class PinnedPrefixState:
    """A pinned-host snapshot (ShadowBoxer/core/caches.py:58-128): the same
    fields, plus the arena that holds them and the event that marks the end
    of their device-to-host copies."""
    prefix_tokens: Tuple[int, ...]
    vision_signature: Tuple[Any, ...]
    prefix_hidden: Optional[torch.Tensor]
    conv_states: Dict[int, torch.Tensor]
    recurrent_states: Dict[int, torch.Tensor]
    key_cache: Dict[int, torch.Tensor]
    value_cache: Dict[int, torch.Tensor]
    rope_deltas: Optional[torch.Tensor]
    available_offsets: Tuple[int, ...] = ()
    conv_checkpoints: Dict[int, Dict[int, torch.Tensor]] = field(default_factory=dict)
    recurrent_checkpoints: Dict[int, Dict[int, torch.Tensor]] = field(default_factory=dict)
    ready: Optional[torch.cuda.Event] = None
    nbytes: int = 0
    _arena: Optional[_PinnedArena] = None

    def is_ready(self) -> bool:
        """True once every device-to-host copy of the snapshot has finished."""
        return self.ready is None or self.ready.query()

    def synchronize(self) -> None:
        if self.ready is not None:
            self.ready.synchronize()

    def resolve_best_offset(self, max_allowed_len: int) -> Optional[int]:
        """Largest restorable offset <= max_allowed_len (caches.py:72-84)."""
        offsets = self.available_offsets if self.available_offsets else (len(self.prefix_tokens),)
        best: Optional[int] = None
        for off in offsets:
            if off <= max_allowed_len and (best is None or off > best):
                best = off
        return best

    def restore(self, device: torch.device, snap_len: Optional[int] = None
                ) -> Tuple[Qwen3_5HybridCache, Optional[torch.Tensor], int]:
        """A new cache at `snap_len` tokens (caches.py:86-128): the checkpoint
        states recorded at that offset, else the current ones; the KV cache and
        the prefix hidden states cut to `snap_len`.  The copies run on the copy
        stream; the caller's current stream waits for them, the host does not."""
        target_len = int(snap_len) if snap_len is not None else len(self.prefix_tokens)
        conv_src = self.conv_checkpoints.get(target_len, self.conv_states)
        rec_src = self.recurrent_checkpoints.get(target_len, self.recurrent_states)
        names: List[Tuple[str, Any]] = []
        host: List[torch.Tensor] = []

        def add(name: str, key: Any, t: Optional[torch.Tensor]) -> None:
            if t is not None:
                names.append((name, key))
                host.append(t)

        add("rope", None, self.rope_deltas)
        for k, v in conv_src.items():
            add("conv", k, v)
        for k, v in rec_src.items():
            add("rec", k, v)
        for k, v in self.key_cache.items():
            add("key", k, v[:, :, :target_len, :] if v.shape[2] > target_len else v)
        for k, v in self.value_cache.items():
            add("value", k, v[:, :, :target_len, :] if v.shape[2] > target_len else v)
        if self.prefix_hidden is not None:
            h = self.prefix_hidden
            add("hidden", None, h[:, :target_len, :] if h.shape[1] > target_len else h)
        outs = _h2d(host, device, self.ready) if host else []
        cache = Qwen3_5HybridCache()
        cache.past_seen_tokens = target_len
        hidden = None
        for (name, key), t in zip(names, outs):
            if name == "rope":
                cache.rope_deltas = t
            elif name == "conv":
                cache.conv_states[key] = t
            elif name == "rec":
                cache.recurrent_states[key] = mark_owned(t if t.dtype == torch.float32 else t.float(), cache, key)
            elif name == "key":
                cache.key_cache[key] = t
            elif name == "value":
                cache.value_cache[key] = t
            else:
                hidden = t
        return cache, hidden, target_len


def snapshot_prefix_state(prefix_tokens: Sequence[int], prefix_hidden: Optional[torch.Tensor],
                          hybrid_cache: Qwen3_5HybridCache, vision_signature: Tuple[Any, ...] = ()
                          ) -> Optional[PinnedPrefixState]:
    """Pinned snapshot of `hybrid_cache` after `prefix_tokens`, with the
    reference's selection rules (caches.py:203-299): checkpoints at
    1 <= cp <= len(prefix_tokens) recorded for both state kinds, the current
    states as the full-length entry, the KV cache and hidden states cut to the
    largest restorable offset.  Returns None when nothing is restorable.  Each
    distinct device tensor is copied once, asynchronously."""
    pfx = tuple(int(x) for x in prefix_tokens)
    full_len = len(pfx)
    if full_len == 0:
        return None
    have_current = bool(hybrid_cache.conv_states or hybrid_cache.recurrent_states)
    offsets = snapshot_offsets(hybrid_cache.conv_checkpoints, hybrid_cache.recurrent_checkpoints, full_len,
                               have_current)
    if not offsets:
        return None
    max_kv = max(offsets)
    conv_cp = {int(cp): dict(m) for cp, m in hybrid_cache.conv_checkpoints.items() if 1 <= int(cp) <= full_len and m}
    rec_cp = {int(cp): dict(m) for cp, m in hybrid_cache.recurrent_checkpoints.items()
              if 1 <= int(cp) <= full_len and m}
    if have_current:
        conv_cp.setdefault(full_len, dict(hybrid_cache.conv_states))
        rec_cp.setdefault(full_len, dict(hybrid_cache.recurrent_states))

    srcs: List[torch.Tensor] = []
    slot: Dict[int, int] = {}  # id(device tensor) -> index in srcs

    def take(t: Optional[torch.Tensor]) -> Optional[int]:
        if t is None:
            return None
        if not t.is_cuda:
            raise RuntimeError("prefix snapshots need CUDA tensors")
        i = slot.get(id(t))
        if i is None:
            i = slot[id(t)] = len(srcs)
            srcs.append(t)
        return i

    plan: Dict[str, Any] = {
        "hidden": take(None if prefix_hidden is None else
                       (prefix_hidden[:, :max_kv, :] if prefix_hidden.shape[1] > max_kv else prefix_hidden)),
        "rope": take(hybrid_cache.rope_deltas),
        "conv": {k: take(v) for k, v in hybrid_cache.conv_states.items()},
        "rec": {k: take(v) for k, v in hybrid_cache.recurrent_states.items()},
        "key": {k: take(v[:, :, :max_kv, :] if v.shape[2] > max_kv else v) for k, v in hybrid_cache.key_cache.items()},
        "value": {k: take(v[:, :, :max_kv, :] if v.shape[2] > max_kv else v)
                  for k, v in hybrid_cache.value_cache.items()},
        "conv_cp": {cp: {k: take(v) for k, v in m.items()} for cp, m in conv_cp.items()},
        "rec_cp": {cp: {k: take(v) for k, v in m.items()} for cp, m in rec_cp.items()},
    }
    arena, done = _d2h(srcs)
    # the copies read these tensors until `done`: the layer must not update them in place
    for t in srcs:
        _release_ownership(t)
    V = arena.views

    def pick(i: Optional[int]) -> Optional[torch.Tensor]:
        return None if i is None else V[i]

    return PinnedPrefixState(
        prefix_tokens=pfx[:max_kv], vision_signature=tuple(vision_signature), prefix_hidden=pick(plan["hidden"]),
        conv_states={k: V[i] for k, i in plan["conv"].items()},
        recurrent_states={k: V[i] for k, i in plan["rec"].items()},
        key_cache={k: V[i] for k, i in plan["key"].items()}, value_cache={k: V[i] for k, i in plan["value"].items()},
        rope_deltas=pick(plan["rope"]), available_offsets=offsets,
        conv_checkpoints={cp: {k: V[i] for k, i in m.items()} for cp, m in plan["conv_cp"].items()},
        recurrent_checkpoints={cp: {k: V[i] for k, i in m.items()} for cp, m in plan["rec_cp"].items()},
        ready=done, nbytes=arena.nbytes, _arena=arena)


class PrefixStateCache:
    """The prefix part of ``PromptEmbedCache`` (caches.py:131-340): an LRU of
    snapshots keyed by (prefix tokens, vision signature)."""

    def __init__(self, max_prefix_entries: int = 8):
        self.max_prefix_entries = int(max_prefix_entries)
        self._prefix_cache: "OrderedDict[Tuple[Any, ...], PinnedPrefixState]" = OrderedDict()
        self.splice_hits = 0

    def __len__(self) -> int:
        return len(self._prefix_cache)

    def insert_prefix_state(self, prefix_tokens: Sequence[int], prefix_hidden: Optional[torch.Tensor],
                            hybrid_cache: Qwen3_5HybridCache, vision_signature: Tuple[Any, ...] = ()
                            ) -> Optional[PinnedPrefixState]:
        st = snapshot_prefix_state(prefix_tokens, prefix_hidden, hybrid_cache, vision_signature)
        if st is None:
            return None
        key: Tuple[Any, ...] = (st.prefix_tokens, st.vision_signature) if st.vision_signature else st.prefix_tokens
        self._prefix_cache[key] = st
        self._prefix_cache.move_to_end(key)
        while len(self._prefix_cache) > self.max_prefix_entries:
            self._prefix_cache.popitem(last=False)
        return st

    def find(self, token_ids: Sequence[int], vision_signature: Tuple[Any, ...] = ()
             ) -> Optional[Tuple[Tuple[Any, ...], PinnedPrefixState, int]]:
        """(key, snapshot, offset) of the longest usable splice, most recent
        first, never the whole prompt (caches.py:301-336); None under 16 tokens."""
        toks = [int(x) for x in token_ids]
        total = len(toks)
        if total < 16 or not self._prefix_cache:
            return None
        best = None
        best_len = 0
        for key, st in reversed(self._prefix_cache.items()):
            if st.vision_signature != tuple(vision_signature):
                continue
            max_allowed = min(common_prefix_len(st.prefix_tokens, toks), total - 1)
            if max_allowed <= best_len:
                continue
            off = st.resolve_best_offset(max_allowed)
            if off is not None and off > best_len:
                best, best_len = (key, st), off
        if best is None or best_len <= 0:
            return None
        return best[0], best[1], best_len

    def lookup_prefix_splice(self, token_ids: Sequence[int], device: torch.device,
                             vision_signature: Tuple[Any, ...] = ()
                             ) -> Optional[Tuple[Qwen3_5HybridCache, Optional[torch.Tensor], int]]:
        hit = self.find(token_ids, vision_signature)
        if hit is None:
            return None
        key, st, off = hit
        self._prefix_cache.move_to_end(key)
        self.splice_hits += 1
        return st.restore(device, snap_len=off)


__all__ = ["PinnedPrefixState", "PrefixStateCache", "snapshot_prefix_state", "snapshot_offsets",
           "common_prefix_len", "copy_stream"]
