"""Hybrid per-layer cache with the reference's layout and checkpoint rules.

Same attribute names, shapes, dtypes and semantics as
``Qwen3_5HybridCache`` (ShadowBoxer/models/qwen35/cache.py:9-244), so the
engine, the prefix cache and speculative-decode rollback see no difference:

* ``conv_states[layer]``      [B, conv_dim, K-1], activation dtype
* ``recurrent_states[layer]`` [B, Hv, dk, dv], float32
* ``conv_checkpoints[pos][layer]`` / ``recurrent_checkpoints[pos][layer]``
  keyed by absolute token position
* ``checkpoint_offsets``      positions the layer snapshots (set by
  ``resolve_active_checkpoints``)
* ``past_seen_tokens``        advanced by the caller, never by the layer

Tensors that the DeltaNet layer allocated for this cache carry an ownership
tag, so a later step may update them in place; anything else placed in the
cache (a restored snapshot, a clone) is treated as shared and never written.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Sequence, Set, Tuple

import torch

_OWNER_ATTR = "_gdn_owned_by"


def mark_owned(t: torch.Tensor, cache: "Qwen3_5HybridCache", layer_idx: int) -> torch.Tensor:
    setattr(t, _OWNER_ATTR, (id(cache), int(layer_idx)))
    return t


def is_owned(t: Optional[torch.Tensor], cache: "Qwen3_5HybridCache", layer_idx: int) -> bool:
    return t is not None and getattr(t, _OWNER_ATTR, None) == (id(cache), int(layer_idx))


class Qwen3_5HybridCache:
    def __init__(self, record_checkpoints: bool = False, checkpoint_positions: Optional[Sequence[int]] = None,
                 min_checkpoint_token: int = 0, structural_checkpoints: Optional[Sequence[int]] = None) -> None:
        self.conv_states: Dict[int, torch.Tensor] = {}
        self.recurrent_states: Dict[int, torch.Tensor] = {}
        self.key_cache: Dict[int, torch.Tensor] = {}
        self.value_cache: Dict[int, torch.Tensor] = {}
        self.past_seen_tokens: int = 0
        self.rope_deltas: Optional[torch.Tensor] = None
        self.record_checkpoints: bool = bool(record_checkpoints)
        self.requested_checkpoints: Optional[Set[int]] = (
            None if checkpoint_positions is None else {int(p) for p in checkpoint_positions})
        self.structural_checkpoints: Set[int] = {int(p) for p in (structural_checkpoints or ())}
        self.min_checkpoint_token: int = int(min_checkpoint_token)
        self.checkpoint_offsets: List[int] = []
        self.conv_checkpoints: Dict[int, Dict[int, torch.Tensor]] = {}
        self.recurrent_checkpoints: Dict[int, Dict[int, torch.Tensor]] = {}

    # ------------------------------------------------------------------
    @staticmethod
    def derive_structural_checkpoints(token_ids: Sequence[int], vision_end_token_id: int = 248054,
                                      im_end_token_id: int = 248046, max_structural: int = 8
                                      ) -> Tuple[int, List[int]]:
        """Anchor positions after vision blocks / turn ends plus a spaced tail
        (cache.py:39-80): returns (min_snap, sorted anchors)."""
        n = len(token_ids)
        min_snap = 0
        anchors: List[int] = []
        for i, tok in enumerate(int(t) for t in token_ids):
            if tok == vision_end_token_id:
                min_snap = i + 1
                anchors.append(i + 1)
            elif tok in (im_end_token_id, 248044) and i + 1 < n and min_snap == 0:
                anchors.append(i + 1)
        lo, hi = max(min_snap, 8), n - 1
        if hi - lo >= 16:
            step = max(12, (hi - lo) // max(2, max_structural))
            pos = ((lo + 3) // 4) * 4
            while pos <= hi:
                anchors.append(pos)
                pos = ((pos + step + 3) // 4) * 4
        uniq = sorted({p for p in anchors if 8 <= p < n})
        if len(uniq) > max_structural:
            stride = len(uniq) / float(max_structural)
            uniq = sorted({uniq[min(len(uniq) - 1, int(round(i * stride)))] for i in range(max_structural)})
        return min_snap, uniq

    def resolve_active_checkpoints(self, past_seen: int, seq_len: int) -> List[int]:
        """Absolute positions to snapshot during the next forward (cache.py:82-129)."""
        if not self.record_checkpoints:
            return []
        total = past_seen + seq_len
        if self.requested_checkpoints is not None:
            lo = max(past_seen + 1, self.min_checkpoint_token)
            self.checkpoint_offsets = sorted(p for p in self.requested_checkpoints if lo <= p <= total)
            return self.checkpoint_offsets
        lo = max(past_seen + 1, self.min_checkpoint_token, 8)
        hi = total - 1
        if lo > hi:
            return []
        span = total - lo
        cands: Set[int] = set()
        if lo <= self.min_checkpoint_token <= hi:
            cands.add(self.min_checkpoint_token)
        cands.update(p for p in self.structural_checkpoints if lo <= p <= hi)
        for frac in (0.25, 0.50, 0.65, 0.75, 0.82, 0.90):
            raw = lo + int(round(span * frac))
            snapped = (raw // 4) * 4
            if lo <= snapped <= hi:
                cands.add(snapped)
            elif lo <= raw <= hi:
                cands.add(raw)
        first = ((lo + 63) // 64) * 64
        cands.update(range(max(64, first), hi + 1, 64))
        self.checkpoint_offsets = sorted(cands)
        return self.checkpoint_offsets

    # ------------------------------------------------------------------
    def extract_checkpoint(self, token_offset: int) -> "Qwen3_5HybridCache":
        """A new cache holding the states recorded at ``token_offset`` (cache.py:131-154)."""
        off = int(token_offset)
        if off == self.past_seen_tokens and off not in self.recurrent_checkpoints:
            return self.clone_and_expand(1)
        if off not in self.conv_checkpoints or off not in self.recurrent_checkpoints:
            raise KeyError(f"Checkpoint offset {off} not recorded in Qwen3_5HybridCache "
                           f"(available: {self.checkpoint_offsets})")
        out = Qwen3_5HybridCache()
        out.past_seen_tokens = off
        if self.rope_deltas is not None:
            out.rope_deltas = self.rope_deltas.clone()
        for k, v in self.conv_checkpoints[off].items():
            out.conv_states[k] = v.contiguous().clone()
        for k, v in self.recurrent_checkpoints[off].items():
            out.recurrent_states[k] = v.contiguous().clone()
        for k, v in self.key_cache.items():
            out.key_cache[k] = v[:, :, :off, :].contiguous().clone()
        for k, v in self.value_cache.items():
            out.value_cache[k] = v[:, :, :off, :].contiguous().clone()
        return out

    def clone_and_expand(self, batch_repeats: int = 1, record_checkpoints: bool = False,
                         checkpoint_positions: Optional[Sequence[int]] = None) -> "Qwen3_5HybridCache":
        """Deep copy with every batch row repeated ``batch_repeats`` times (cache.py:156-197)."""
        out = Qwen3_5HybridCache(record_checkpoints=record_checkpoints, checkpoint_positions=checkpoint_positions)
        out.past_seen_tokens = int(self.past_seen_tokens)
        r = int(batch_repeats)

        def rep(v: torch.Tensor) -> torch.Tensor:
            if r > 1:
                return v.repeat(r, *([1] * (v.dim() - 1))).contiguous()
            return v.clone()

        if self.rope_deltas is not None:
            out.rope_deltas = rep(self.rope_deltas)
        for src, dst in ((self.conv_states, out.conv_states), (self.recurrent_states, out.recurrent_states),
                         (self.key_cache, out.key_cache), (self.value_cache, out.value_cache)):
            for k, v in src.items():
                dst[k] = rep(v)
        return out

    def select_batch_item(self, batch_idx: int, total_valid_tokens: Optional[int] = None) -> "Qwen3_5HybridCache":
        """Row ``batch_idx`` rolled back to ``total_valid_tokens`` (cache.py:199-244).

        With no checkpoint recorded at that position the current states are
        used, as in the reference."""
        out = Qwen3_5HybridCache()
        target = int(total_valid_tokens) if total_valid_tokens is not None else int(self.past_seen_tokens)
        out.past_seen_tokens = target
        if self.rope_deltas is not None:
            i = min(batch_idx, self.rope_deltas.shape[0] - 1)
            out.rope_deltas = self.rope_deltas[i:i + 1].clone()
        use_cp = total_valid_tokens is not None
        conv_src = self.conv_checkpoints[target] if use_cp and target in self.conv_checkpoints else self.conv_states
        rec_src = (self.recurrent_checkpoints[target] if use_cp and target in self.recurrent_checkpoints
                   else self.recurrent_states)
        sl = slice(batch_idx, batch_idx + 1)
        for k, v in conv_src.items():
            out.conv_states[k] = v[sl].contiguous().clone()
        for k, v in rec_src.items():
            out.recurrent_states[k] = v[sl].contiguous().clone()
        for src, dst in ((self.key_cache, out.key_cache), (self.value_cache, out.value_cache)):
            for k, v in src.items():
                s = v[sl]
                if use_cp:
                    s = s[:, :, :target, :]
                dst[k] = s.contiguous().clone()
        return out


__all__ = ["Qwen3_5HybridCache", "mark_owned", "is_owned"]
