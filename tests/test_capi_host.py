"""The C-ABI library: it loads without a GPU, exports every declared entry
point, and rejects bad arguments on the host (no launch happens in any case
below: every call carries at least one invalid field)."""
from __future__ import annotations

import ctypes
import json
import os
import re

import pytest
import torch

from visionstack_b200 import Qwen3_5GatedDeltaNet, Qwen3_5TextConfig, _lib

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "gdn_b200.h")


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(gdn_\w+)\s*\(", text, re.M)))


def test_header_declares_the_bound_symbols():
    assert declared_functions() == sorted(_lib.EXPORTED_SYMBOLS)


def test_library_loads_and_exports_every_symbol():
    lib = _lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert lib.gdn_version() == 1


def _valid_args(T=1):
    """Arguments that would pass validation; tests break one field each."""
    a = _lib.MixerArgs()
    a.batch, a.seq_len, a.num_k_heads, a.num_v_heads = 2, T, 2, 4
    a.head_k_dim = a.head_v_dim = 32
    a.conv_kernel, a.act_dtype, a.norm_eps = 4, _lib.GDN_DTYPE_BF16, 1e-6
    conv_dim = 2 * 2 * 32 + 4 * 32
    a.mixed_qkv, a.mixed_stride_b, a.mixed_stride_t = 0x10000, T * conv_dim, conv_dim
    a.z, a.z_stride_b, a.z_stride_t = 0x20000, T * 128, 128
    a.a, a.b, a.ab_stride_b, a.ab_stride_t = 0x30000, 0x31000, T * 4, 4
    a.conv_weight, a.A_log, a.dt_bias, a.norm_weight = 0x40000, 0x41000, 0x42000, 0x43000
    a.out = 0x50000
    a.state_in = a.state_out = 0x60000
    return a


def _call(fn, args):
    lib = _lib.load()
    return getattr(lib, fn)(ctypes.byref(args), None)


@pytest.mark.parametrize("fn", ["gdn_mixer_decode", "gdn_mixer_prefill"])
@pytest.mark.parametrize("breaker,code", [
    (lambda a: setattr(a, "batch", 0), -1),
    (lambda a: setattr(a, "num_v_heads", 3), -1),
    (lambda a: setattr(a, "head_v_dim", 48), -2),
    (lambda a: setattr(a, "head_k_dim", 256), -2),
    (lambda a: setattr(a, "conv_kernel", 5), -2),
    (lambda a: setattr(a, "act_dtype", 7), -2),
    (lambda a: setattr(a, "mixed_qkv", None), -1),
    (lambda a: setattr(a, "mixed_stride_t", 10), -1),
    (lambda a: setattr(a, "z_stride_t", 3), -1),
    (lambda a: setattr(a, "state_in", 0x60004), -3),
    (lambda a: setattr(a, "out", 0x50001), -3),
    (lambda a: (setattr(a, "conv_state_in", 0x70000), setattr(a, "conv_state_out", 0x70000)), -1),
])
def test_mixer_validation(fn, breaker, code):
    a = _valid_args()
    breaker(a)
    assert _call(fn, a) == code
    assert _lib.load().gdn_last_error_string()


def test_checkpoint_validation():
    a = _valid_args(T=4)
    offs = _lib.int_array([1, 2, 2])
    a.num_checkpoints = 3
    a.checkpoint_offsets = ctypes.cast(offs, ctypes.POINTER(ctypes.c_int32))
    a.state_checkpoints, a.conv_checkpoints = 0x80000, 0x90000
    assert _call("gdn_mixer_decode", a) == -1  # duplicate offset
    a.num_checkpoints = _lib.GDN_MAX_CHECKPOINTS + 1
    assert _call("gdn_mixer_prefill", a) == -5
    a.num_checkpoints = 2
    a.state_checkpoints = None
    assert _call("gdn_mixer_decode", a) == -1  # slots requested without buffers


def test_decode_rejects_long_sequences():
    a = _valid_args(T=9)
    a.batch = -1  # also invalid, so nothing can launch
    assert _call("gdn_mixer_decode", a) == -1


def _slot_args(T=4):
    a = _valid_args(T)
    a.state_out = None
    a.conv_state_in = 0x70000
    return a


@pytest.mark.parametrize("breaker,table,n,code", [
    (lambda a: None, None, 5, -1),                              # no slot table
    (lambda a: None, 0xA0002, 5, -3),                           # misaligned table
    (lambda a: None, 0xA0000, 4, -1),                           # fewer than T + 1 slots
    (lambda a: None, 0xA0000, 10, -1),                          # more than 9 slots
    (lambda a: setattr(a, "state_out", 0x60000), 0xA0000, 5, -1),
    (lambda a: setattr(a, "conv_state_in", None), 0xA0000, 5, -1),
    (lambda a: setattr(a, "num_checkpoints", 1), 0xA0000, 5, -1),
    (lambda a: setattr(a, "flags", _lib.GDN_FLAG_REGISTER_KERNEL), 0xA0000, 5, -2),
    (lambda a: setattr(a, "seq_len", 9), 0xA0000, 9, -1),
    (lambda a: setattr(a, "head_k_dim", 256), 0xA0000, 5, -2),
])
def test_verify_slots_validation(breaker, table, n, code):
    a = _slot_args()
    breaker(a)
    assert _lib.load().gdn_mixer_verify_slots(ctypes.byref(a), table, n, None) == code
    assert _lib.load().gdn_last_error_string()


def test_accept_slots_validation():
    lib = _lib.load()
    assert lib.gdn_accept_slots(None, 0xA0000, 4, 5, 4, None) == -1
    assert lib.gdn_accept_slots(0xB0000, 0xA0000, 0, 5, 4, None) == -1
    assert lib.gdn_accept_slots(0xB0000, 0xA0000, 4, 4, 4, None) == -1
    assert lib.gdn_accept_slots(0xB0000, 0xA0000, 4, 5, 0, None) == -1
    assert lib.gdn_accept_slots(0xB0001, 0xA0000, 4, 5, 4, None) == -3


def test_error_raises_runtime_error():
    with pytest.raises(_lib.GDNError):
        _lib.check("gdn_mixer_decode", _call("gdn_mixer_decode", _lib.MixerArgs()))


def test_functional_validation():
    lib = _lib.load()
    assert lib.gdn_delta_rule(1, 4, 2, 48, 48, 0, 16, 16, 16, 16, 16, None, None, 16, 1, 1, 0, None, None,
                              None) == -2
    assert lib.gdn_delta_rule(0, 4, 2, 32, 32, 0, 16, 16, 16, 16, 16, None, None, 16, 1, 1, 0, None, None,
                              None) == -1
    assert lib.gdn_causal_conv1d(1, 8, 4, 6, 0, 16, 16, None, 16, None, 1, None) == -2
    assert lib.gdn_causal_conv1d(1, 8, 4, 4, 1, 17, 16, None, 16, None, 1, None) == -3
    # triangular solve: sizes, the identity needs m == n, alignment, out overlapping ut
    p = 0x100000
    assert lib.gdn_solve_unit_lower_triangular(p, p + 0x10000, p + 0x20000, 0, 64, 8, None) == -1
    assert lib.gdn_solve_unit_lower_triangular(p, None, p + 0x20000, 2, 64, 8, None) == -1
    assert lib.gdn_solve_unit_lower_triangular(p + 2, None, p + 0x20000, 2, 64, 64, None) == -3
    assert lib.gdn_solve_unit_lower_triangular(p, None, p + 64, 2, 64, 64, None) == -1
    assert b"overlap" in lib.gdn_last_error_string()
    # gated norm: dtype codes, NULL pointers, misaligned bf16 rows
    assert lib.gdn_rms_norm_gated(p, p, p, p, 4, 128, 1e-6, 7, 1, 1, None) == -2
    assert lib.gdn_rms_norm_gated(p, None, p, p, 4, 128, 1e-6, 1, 1, 1, None) == -1
    assert lib.gdn_rms_norm_gated(p + 1, p, p, p, 4, 128, 1e-6, 1, 1, 1, None) == -3
    assert lib.gdn_rms_norm_gated(p, p, p, p, 0, 128, 1e-6, 1, 1, 1, None) == -1


def test_functional_names_of_the_reference_module_are_exported():
    import visionstack_b200.deltanet as D
    for name in ("_causal_conv1d_fn", "_chunk_gated_delta_rule", "_recurrent_gated_delta_rule",
                 "_solve_unit_lower_triangular", "_invert_unit_lower_triangular_block"):
        assert name in D.__all__ and callable(getattr(D, name))
    with pytest.raises(RuntimeError, match="CUDA"):
        D._solve_unit_lower_triangular(torch.eye(4), torch.ones(4, 2))


def test_state_dict_matches_reference_layout():
    with open(os.path.join(REPO, "tests", "golden", "cache.json")) as f:
        ref = json.load(f)["state_dict"]
    m = Qwen3_5GatedDeltaNet(Qwen3_5TextConfig(hidden_size=2048), 3)
    ours = {k: list(v.shape) for k, v in m.state_dict().items()}
    assert ours == ref


def test_layer_refuses_cpu_tensors():
    m = Qwen3_5GatedDeltaNet(Qwen3_5TextConfig(hidden_size=64, linear_num_key_heads=1, linear_num_value_heads=2,
                                               linear_key_head_dim=32, linear_value_head_dim=32), 0)
    with pytest.raises(RuntimeError, match="CUDA"):
        m(torch.zeros(1, 3, 64))


def test_attn_decode_validation():
    lib = _lib.load()
    assert lib.gdn_attn_decode_workspace_bytes(32, 2, 8, 256, 4352) > 0
    assert lib.gdn_attn_decode_workspace_bytes(32, 2, 3, 256, 4352) == -1  # groups not in {1, 2, 4, 8}
    assert lib.gdn_attn_decode_workspace_bytes(32, 2, 8, 96, 4352) == -1   # head_dim
    n = lib.gdn_attn_decode_workspace_bytes(2, 2, 8, 256, 64)
    p = 0x100000
    # NULL pointer, misaligned pointer, short workspace: rejected on the host, nothing launches
    assert lib.gdn_attn_decode(0, p, p, p, p, 2, 2, 8, 256, 64, 0.0625, p, n, None) == -1
    assert lib.gdn_attn_decode(p + 2, p, p, p, p, 2, 2, 8, 256, 64, 0.0625, p, n, None) < 0
    assert lib.gdn_attn_decode(p, p, p, p, p, 2, 2, 8, 256, 64, 0.0625, p, n - 16, None) == -1
    assert lib.gdn_last_error_string()


def test_peer_allreduce_validation():
    """The peer all-reduce's size rules and argument checks, on the host (nothing launches)."""
    import ctypes
    lib = _lib.load()
    assert lib.gdn_peer_staging_bytes(2, 32, 1 << 20) >= 4 * (1 << 20)
    assert lib.gdn_peer_staging_bytes(9, 32, 1024) == -1   # more ranks than GDN_PEER_MAX_RANKS
    assert lib.gdn_peer_staging_bytes(2, 0, 1024) == -1    # no blocks
    assert lib.gdn_peer_staging_bytes(2, 32, 1001) == -1   # capacity not a multiple of 8
    ptr = ctypes.c_void_p()
    assert lib.gdn_peer_staging_alloc(0, ctypes.byref(ptr)) == -1
    assert lib.gdn_ipc_get_handle(None, ctypes.create_string_buffer(64)) == -1
    assert lib.gdn_ipc_open_handle(None, ctypes.byref(ptr)) == -1
    g = _lib.PeerGroup()
    g.rank, g.world, g.nblocks, g.cap = 0, 2, 32, 1024
    g.staging[0], g.staging[1] = 0x100000, 0x200000
    p = 0x300000
    call = lambda x, y, n: lib.gdn_peer_allreduce_bf16(ctypes.byref(g), x, y, n, None)  # noqa: E731
    assert lib.gdn_peer_allreduce_bf16(None, p, p, 8, None) == -1
    assert call(p, p, 12) == -1          # not a multiple of 8
    assert call(p, p, 2048) == -1        # above the capacity
    assert call(p + 2, p, 8) == -3       # misaligned
    assert call(p, p, 0) == 0            # nothing to sum
    g.rank = 2
    assert call(p, p, 8) == -1           # rank outside the group
    g.rank = 0
    g.staging[1] = None
    assert call(p, p, 8) == -1           # a rank's staging memory is missing
    assert b"staging" in lib.gdn_last_error_string()


def test_stack_ops_validation():
    lib = _lib.load()
    p = 0x100000
    assert lib.gdn_rms_norm_zc(None, 2048, None, 0, None, p, p, 4, 2048, 1e-6, None) == -1
    assert lib.gdn_rms_norm_zc(p, 2048, p, 2048, None, p, p, 4, 2048, 1e-6, None) == -1   # delta without res_out
    assert lib.gdn_rms_norm_zc(p, 2048, None, 0, None, p, p, 4, 2044, 1e-6, None) == -1   # dim not a multiple of 8
    assert lib.gdn_rms_norm_zc(p, 1024, None, 0, None, p, p, 4, 2048, 1e-6, None) == -1   # stride below dim
    assert lib.gdn_rms_norm_zc(p + 2, 2048, None, 0, None, p, p, 4, 2048, 1e-6, None) == -3
    assert lib.gdn_rms_norm_zc(p, 2048, None, 0, None, p, p, 0, 2048, 1e-6, None) == 0    # no rows
    assert lib.gdn_silu_mul(p, p, p, 12, None) == -1
    assert lib.gdn_silu_mul(p, p + 8, p, 16, None) == -3
    assert lib.gdn_silu_mul(p, p, p, 0, None) == 0
    # attention steps: head_dim / rotary_dim limits, NULL / misaligned pointers
    args = [p] * 8
    assert lib.gdn_qk_norm_rope(*args, 2, 3, 4, 2, 512, 64, 1e-6, None) == -2
    assert lib.gdn_qk_norm_rope(*args, 2, 3, 4, 2, 256, 24, 1e-6, None) == -2
    assert lib.gdn_qk_norm_rope(None, *args[1:], 2, 3, 4, 2, 256, 64, 1e-6, None) == -1
    assert lib.gdn_qk_norm_rope(*args, 0, 3, 4, 2, 256, 64, 1e-6, None) == 0   # no rows
    assert lib.gdn_attn_gate_out(p, 8, 8, 4, p, p, 2, 3, 4, 256, None) == -3  # stride not a multiple of 8
    assert lib.gdn_attn_gate_out(p, 8, 8, 8, p, p, 0, 3, 4, 256, None) == 0   # no rows
    assert lib.gdn_rms_norm_zc(p, 2048, None, 0, None, p, p, 1 << 31, 2048, 1e-6, None) == -1  # grid limit
