"""B200 (sm_100a) Gated DeltaNet token mixer with the reference layer's interface.

Public names mirror ShadowBoxer/models/qwen35 (deltanet.py, cache.py,
config.py).  Kernels live in ``libgdn_b200.so`` (C ABI: include/gdn_b200.h),
loaded on first use; there is no CPU implementation in this package.
"""
from .cache import Qwen3_5HybridCache
from .config import Qwen3_5RMSNormGated, Qwen3_5TextConfig
from .deltanet import (
    Qwen3_5GatedDeltaNet,
    _causal_conv1d_fn,
    _chunk_gated_delta_rule,
    _extract_conv_state_at_offset,
    _invert_unit_lower_triangular_block,
    _recurrent_gated_delta_rule,
    _solve_unit_lower_triangular,
)
from .prefix import PinnedPrefixState, PrefixStateCache, snapshot_prefix_state
from .slots import StateSlots

__all__ = [
    "Qwen3_5HybridCache",
    "Qwen3_5RMSNormGated",
    "Qwen3_5TextConfig",
    "Qwen3_5GatedDeltaNet",
    "StateSlots",
    "PinnedPrefixState",
    "PrefixStateCache",
    "snapshot_prefix_state",
    "_causal_conv1d_fn",
    "_chunk_gated_delta_rule",
    "_extract_conv_state_at_offset",
    "_invert_unit_lower_triangular_block",
    "_recurrent_gated_delta_rule",
    "_solve_unit_lower_triangular",
]
