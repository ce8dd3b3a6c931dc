"""ctypes binding of ``libgdn_b200.so`` (the C ABI in ``include/gdn_b200.h``).

The binding style follows the reference's own native DLL binding: ctypes,
``int32`` status returns, and a non-zero status raised as ``RuntimeError``
with the library's last error string (VizInjector/python/bindings.py:298-400,
551-729).  There is no fallback: if the library is missing or cannot be
loaded, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libgdn_b200.so")

GDN_OK = 0
GDN_DTYPE_F32 = 0
GDN_DTYPE_BF16 = 1
GDN_MAX_CHECKPOINTS = 512
GDN_MAX_DECODE_TOKENS = 8

EXPORTED_SYMBOLS = (
    "gdn_version",
    "gdn_last_error_string",
    "gdn_mixer_decode",
    "gdn_mixer_prefill",
    "gdn_delta_rule",
    "gdn_causal_conv1d",
    "gdn_mixer_verify_slots",
    "gdn_prefill_workspace_bytes",
    "gdn_mixer_prefill_ws",
    "gdn_mixer_prefill_noalloc",
    "gdn_accept_slots",
    "gdn_device_error",
    "gdn_selftest_umma",
    "gdn_selftest_expired_wait",
    "gdn_attn_decode_workspace_bytes",
    "gdn_attn_decode",
    "gdn_solve_unit_lower_triangular",
    "gdn_rms_norm_gated",
    "gdn_peer_staging_bytes",
    "gdn_peer_staging_alloc",
    "gdn_peer_staging_free",
    "gdn_ipc_get_handle",
    "gdn_ipc_open_handle",
    "gdn_ipc_close_handle",
    "gdn_peer_allreduce_bf16",
    "gdn_rms_norm_zc",
    "gdn_silu_mul",
    "gdn_qk_norm_rope",
    "gdn_attn_gate_out",
)
GDN_FLAG_REGISTER_KERNEL = 1
GDN_FLAG_CUDA_CORE_PREFILL = 2
GDN_FLAG_PREP_IN_KERNEL_PREFILL = 4
GDN_DEVERR_TMA_TIMEOUT = 0x1
GDN_DEVERR_BAD_SLOT = 0x4
GDN_DEVERR_HANDOFF_TIMEOUT = 0x8
GDN_DEVERR_PEER_TIMEOUT = 0x10
GDN_IPC_HANDLE_BYTES = 64
GDN_PEER_MAX_RANKS = 8
GDN_STATIC_SCRATCH_BYTES = 64 << 20

_c_void_p = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64


class MixerArgs(ctypes.Structure):
    """Mirror of ``gdn_mixer_args`` (include/gdn_b200.h)."""

    _fields_ = [
        ("batch", _i32), ("seq_len", _i32), ("num_k_heads", _i32), ("num_v_heads", _i32),
        ("head_k_dim", _i32), ("head_v_dim", _i32), ("conv_kernel", _i32), ("act_dtype", _i32),
        ("norm_eps", ctypes.c_float), ("flags", _i32),
        ("mixed_qkv", _c_void_p), ("mixed_stride_b", _i64), ("mixed_stride_t", _i64),
        ("z", _c_void_p), ("z_stride_b", _i64), ("z_stride_t", _i64),
        ("a", _c_void_p), ("b", _c_void_p), ("ab_stride_b", _i64), ("ab_stride_t", _i64),
        ("conv_weight", _c_void_p), ("A_log", _c_void_p), ("dt_bias", _c_void_p), ("norm_weight", _c_void_p),
        ("conv_state_in", _c_void_p), ("conv_state_out", _c_void_p),
        ("state_in", _c_void_p), ("state_out", _c_void_p), ("out", _c_void_p),
        ("num_checkpoints", _i32), ("reserved1", _i32),
        ("checkpoint_offsets", ctypes.POINTER(_i32)),
        ("state_checkpoints", _c_void_p), ("conv_checkpoints", _c_void_p),
    ]


class PeerGroup(ctypes.Structure):
    """Mirror of ``gdn_peer_group`` (include/gdn_b200.h)."""
    _fields_ = [("rank", _i32), ("world", _i32), ("nblocks", _i32), ("cap", _i64),
                ("staging", _c_void_p * GDN_PEER_MAX_RANKS)]


class GDNError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, fn: str, status: int, message: str):
        super().__init__(f"{fn} failed with status {status}: {message}")
        self.status = status


_lock = threading.Lock()
_lib: Optional[ctypes.CDLL] = None


def lib_path() -> str:
    return LIB_PATH


def load() -> ctypes.CDLL:
    """Load the shared library once; raise loudly when it is not there."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m visionstack_b200.build` "
                "(nvcc, sm_100a). There is no fallback implementation.")
        lib = ctypes.CDLL(LIB_PATH)
        lib.gdn_version.restype = _i32
        lib.gdn_version.argtypes = []
        lib.gdn_last_error_string.restype = ctypes.c_char_p
        lib.gdn_last_error_string.argtypes = []
        lib.gdn_mixer_decode.restype = _i32
        lib.gdn_mixer_decode.argtypes = [ctypes.POINTER(MixerArgs), _c_void_p]
        lib.gdn_mixer_prefill.restype = _i32
        lib.gdn_mixer_prefill.argtypes = [ctypes.POINTER(MixerArgs), _c_void_p]
        lib.gdn_delta_rule.restype = _i32
        lib.gdn_delta_rule.argtypes = [_i32, _i32, _i32, _i32, _i32, _i32, _c_void_p, _c_void_p, _c_void_p,
                                       _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i32,
                                       ctypes.POINTER(_i32), _c_void_p, _c_void_p]
        lib.gdn_causal_conv1d.restype = _i32
        lib.gdn_causal_conv1d.argtypes = [_i32, _i32, _i32, _i32, _i32, _c_void_p, _c_void_p, _c_void_p,
                                          _c_void_p, _c_void_p, _i32, _c_void_p]
        lib.gdn_selftest_umma.restype = _i32
        lib.gdn_selftest_umma.argtypes = [_i32, _c_void_p, _c_void_p, _c_void_p, _c_void_p]
        lib.gdn_selftest_expired_wait.restype = _i32
        lib.gdn_selftest_expired_wait.argtypes = [_i32, _c_void_p, _c_void_p]
        lib.gdn_attn_decode_workspace_bytes.restype = _i64
        lib.gdn_attn_decode_workspace_bytes.argtypes = [_i32, _i32, _i32, _i32, _i32]
        lib.gdn_attn_decode.restype = _i32
        lib.gdn_attn_decode.argtypes = [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i32,
                                        _i32, _i32, ctypes.c_float, _c_void_p, _i64, _c_void_p]
        lib.gdn_prefill_workspace_bytes.restype = _i64
        lib.gdn_prefill_workspace_bytes.argtypes = [ctypes.POINTER(MixerArgs)]
        lib.gdn_mixer_prefill_ws.restype = _i32
        lib.gdn_mixer_prefill_ws.argtypes = [ctypes.POINTER(MixerArgs), _c_void_p, _i64, _c_void_p]
        lib.gdn_mixer_prefill_noalloc.restype = _i32
        lib.gdn_mixer_prefill_noalloc.argtypes = [ctypes.POINTER(MixerArgs), _c_void_p]
        lib.gdn_mixer_verify_slots.restype = _i32
        lib.gdn_mixer_verify_slots.argtypes = [ctypes.POINTER(MixerArgs), _c_void_p, _i32, _c_void_p]
        lib.gdn_accept_slots.restype = _i32
        lib.gdn_accept_slots.argtypes = [_c_void_p, _c_void_p, _i32, _i32, _i32, _c_void_p]
        lib.gdn_solve_unit_lower_triangular.restype = _i32
        lib.gdn_solve_unit_lower_triangular.argtypes = [_c_void_p, _c_void_p, _c_void_p, _i64, _i32, _i32, _c_void_p]
        lib.gdn_rms_norm_gated.restype = _i32
        lib.gdn_rms_norm_gated.argtypes = [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i32, ctypes.c_float,
                                           _i32, _i32, _i32, _c_void_p]
        lib.gdn_peer_staging_bytes.restype = _i64
        lib.gdn_peer_staging_bytes.argtypes = [_i32, _i32, _i64]
        lib.gdn_peer_staging_alloc.restype = _i32
        lib.gdn_peer_staging_alloc.argtypes = [_i64, ctypes.POINTER(_c_void_p)]
        lib.gdn_peer_staging_free.restype = _i32
        lib.gdn_peer_staging_free.argtypes = [_c_void_p]
        lib.gdn_ipc_get_handle.restype = _i32
        lib.gdn_ipc_get_handle.argtypes = [_c_void_p, _c_void_p]
        lib.gdn_ipc_open_handle.restype = _i32
        lib.gdn_ipc_open_handle.argtypes = [_c_void_p, ctypes.POINTER(_c_void_p)]
        lib.gdn_ipc_close_handle.restype = _i32
        lib.gdn_ipc_close_handle.argtypes = [_c_void_p]
        lib.gdn_peer_allreduce_bf16.restype = _i32
        lib.gdn_peer_allreduce_bf16.argtypes = [ctypes.POINTER(PeerGroup), _c_void_p, _c_void_p, _i64, _c_void_p]
        lib.gdn_rms_norm_zc.restype = _i32
        lib.gdn_rms_norm_zc.argtypes = [_c_void_p, _i64, _c_void_p, _i64, _c_void_p, _c_void_p, _c_void_p, _i64, _i32,
                                        ctypes.c_float, _c_void_p]
        lib.gdn_silu_mul.restype = _i32
        lib.gdn_silu_mul.argtypes = [_c_void_p, _c_void_p, _c_void_p, _i64, _c_void_p]
        lib.gdn_qk_norm_rope.restype = _i32
        lib.gdn_qk_norm_rope.argtypes = [_c_void_p] * 8 + [_i32] * 6 + [ctypes.c_float, _c_void_p]
        lib.gdn_attn_gate_out.restype = _i32
        lib.gdn_attn_gate_out.argtypes = [_c_void_p, _i64, _i64, _i64, _c_void_p, _c_void_p, _i32, _i32, _i32, _i32,
                                          _c_void_p]
        lib.gdn_device_error.restype = _i32
        lib.gdn_device_error.argtypes = [ctypes.POINTER(ctypes.c_uint32), _i32]
        _lib = lib
        return lib


def check(fn: str, status: int) -> None:
    if status != GDN_OK:
        msg = load().gdn_last_error_string()
        raise GDNError(fn, int(status), msg.decode(errors="replace") if msg else "")


def device_error(clear: bool = True) -> int:
    """Sticky device error bits (bounded waits that gave up); synchronises."""
    v = ctypes.c_uint32(0)
    check("gdn_device_error", load().gdn_device_error(ctypes.byref(v), 1 if clear else 0))
    return int(v.value)


def int_array(values) -> "ctypes.Array":
    vals = [int(v) for v in values]
    return (_i32 * max(1, len(vals)))(*vals)
