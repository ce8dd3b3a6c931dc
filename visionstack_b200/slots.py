"""Per-row state slots of one Gated DeltaNet layer for speculative decoding.

The reference verifies a T-token draft on a cache cloned for the candidates
(``Qwen3_5HybridCache.clone_and_expand``, ShadowBoxer/models/qwen35/cache.py:156-197)
with a checkpoint after every draft token, then restores the state of the
accepted length by copying it out of the checkpoint dicts
(``select_batch_item``, cache.py:199-244; ``extract_checkpoint``,
cache.py:131-154; the loop at ShadowBoxer/models/qwen35/speculative.py:778-882).

``StateSlots`` keeps ``draft_len + 1`` state slots per batch row instead.  The
verify kernel (``Qwen3_5GatedDeltaNet.mixer_verify`` -> gdn_mixer_verify_slots)
reads each row's current slot and writes the states after 1..T draft tokens
into the row's other slots; accepting ``a`` tokens (``accept``, ->
gdn_accept_slots) swaps two entries of the row's slot table on the device.  No
state is cloned or copied per step, and the accepted counts never visit the
host.  Accepting 0 tokens keeps the state from before the draft.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from . import _lib


class StateSlots:
    """``num_slots = draft_len + 1`` recurrent / conv state slots per row.

    state  [num_slots, B, Hv, dk, dv] float32
    conv   [num_slots, B, conv_dim, K-1] activation dtype
    table  [B, num_slots] int32: table[b, 0] is row b's current slot, the
           other columns its free slots; after a verify of T tokens, column t
           holds the state after t draft tokens.
    """

    def __init__(self, layer, batch: int, draft_len: int, dtype: torch.dtype = torch.bfloat16,
                 device: Optional[torch.device] = None):
        if not 1 <= draft_len <= _lib.GDN_MAX_DECODE_TOKENS:
            raise ValueError(f"draft_len {draft_len} outside 1..{_lib.GDN_MAX_DECODE_TOKENS}")
        device = torch.device(device if device is not None else "cuda")
        n = draft_len + 1
        self.batch, self.draft_len, self.num_slots = batch, draft_len, n
        self.state = torch.zeros((n, batch, layer.num_v_heads, layer.head_k_dim, layer.head_v_dim),
                                 dtype=torch.float32, device=device)
        self.conv = torch.zeros((n, batch, layer.conv_dim, layer.conv_kernel_size - 1), dtype=dtype, device=device)
        self.table = torch.arange(n, dtype=torch.int32, device=device).repeat(batch, 1).contiguous()
        self._rows = torch.arange(batch, device=device)
        self.last_len = 0

    def _cols(self, col: int) -> torch.Tensor:
        return self.table[:, col].long()

    def load(self, conv_state: Optional[torch.Tensor] = None, rec_state: Optional[torch.Tensor] = None) -> None:
        """Set every row's current state (zeros where None), e.g. from a
        prefilled ``Qwen3_5HybridCache`` entry."""
        cur = self._cols(0)
        self.state[cur, self._rows] = 0.0 if rec_state is None else rec_state.to(self.state)
        self.conv[cur, self._rows] = 0.0 if conv_state is None else conv_state.to(self.conv)

    def current(self) -> Tuple[torch.Tensor, torch.Tensor]:
        """(conv state [B, conv_dim, K-1], recurrent state [B, Hv, dk, dv]) of
        every row's current slot, as new tensors."""
        cur = self._cols(0)
        return self.conv[cur, self._rows], self.state[cur, self._rows]

    def after(self, t: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """States after ``t`` tokens of the last verify (before ``accept``);
        t = 0 is the starting state."""
        if not 0 <= t <= self.last_len:
            raise KeyError(f"no state after {t} tokens (last draft had {self.last_len})")
        col = self._cols(t)
        return self.conv[col, self._rows], self.state[col, self._rows]

    def accept(self, accepted: torch.Tensor) -> None:
        """Row b continues from its state after ``accepted[b]`` draft tokens
        (device tensor [B], 0..T of the last verify)."""
        if self.last_len < 1:
            raise RuntimeError("accept() before any verify")
        if accepted.shape != (self.batch,) or accepted.device != self.table.device:
            raise ValueError("accepted must be a [batch] tensor on the slots' device")
        acc = accepted if accepted.dtype == torch.int32 else accepted.to(torch.int32)
        acc = acc.contiguous()
        dev = self.table.device
        with torch.cuda.device(dev):
            _lib.check("gdn_accept_slots",
                       _lib.load().gdn_accept_slots(acc.data_ptr(), self.table.data_ptr(), self.batch, self.num_slots,
                                                    self.last_len, torch.cuda.current_stream(dev).cuda_stream))


__all__ = ["StateSlots"]
