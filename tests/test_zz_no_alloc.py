"""gdn_mixer_prefill_noalloc: the chunked prefill with its scratch in the
library's fixed device array (no allocation in the call), for C / FFI callers
that have no device allocator.  Compared, bit for bit, with
gdn_mixer_prefill_ws (workspace from torch's allocator) on two calls in a row
with different inputs, once with fewer (batch, head) chains than SMs and once
with more (160 chains: the sequential pass then cuts the chains into runs with
state hand-offs through flags in the shared scratch, which every call must
clear again); oversize calls are rejected.  This file is collected last so
that it also runs after every other test has used the library on the same
device."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from visionstack_b200 import _lib
from visionstack_b200 import workloads as W


def _fake_args(B: int, T: int):
    """Valid-looking arguments with fake aligned device pointers (never launched)."""
    s = W.SHAPE_QWEN
    a = _lib.MixerArgs()
    a.batch, a.seq_len, a.num_k_heads, a.num_v_heads = B, T, s.num_k_heads, s.num_v_heads
    a.head_k_dim = a.head_v_dim = 128
    a.conv_kernel, a.act_dtype, a.norm_eps = 4, _lib.GDN_DTYPE_BF16, 1e-6
    a.mixed_qkv, a.mixed_stride_b, a.mixed_stride_t = 0x100000, T * s.conv_dim, s.conv_dim
    a.z, a.z_stride_b, a.z_stride_t = 0x200000, T * s.value_dim, s.value_dim
    a.a, a.b, a.ab_stride_b, a.ab_stride_t = 0x300000, 0x310000, T * s.num_v_heads, s.num_v_heads
    a.conv_weight, a.A_log, a.dt_bias, a.norm_weight = 0x400000, 0x410000, 0x420000, 0x430000
    a.out = 0x500000
    return a


def test_noalloc_rejects_calls_larger_than_the_static_scratch():
    lib = _lib.load()
    # the prep-in-kernel prefill needs at most one hand-off state per SM, at any length
    fused = _fake_args(8, 8192)
    fused.flags = _lib.GDN_FLAG_PREP_IN_KERNEL_PREFILL
    assert 0 <= lib.gdn_prefill_workspace_bytes(ctypes.byref(fused)) <= 148 * (64 << 10) + 4096
    # the default two-kernel form keeps every chunk's preparation in the workspace: far beyond the scratch
    big = _fake_args(8, 8192)
    need = lib.gdn_prefill_workspace_bytes(ctypes.byref(big))
    assert need > _lib.GDN_STATIC_SCRATCH_BYTES
    assert lib.gdn_mixer_prefill_noalloc(ctypes.byref(big), None) == -1
    assert b"static scratch" in lib.gdn_last_error_string()
    small = _fake_args(1, 512)
    assert 0 < lib.gdn_prefill_workspace_bytes(ctypes.byref(small)) <= _lib.GDN_STATIC_SCRATCH_BYTES
    bad = _fake_args(1, 512)
    bad.batch = 0
    assert lib.gdn_mixer_prefill_noalloc(ctypes.byref(bad), None) == -1


@pytest.mark.gpu
@pytest.mark.parametrize("flags", [0, _lib.GDN_FLAG_PREP_IN_KERNEL_PREFILL], ids=["two_kernel", "prep_in_kernel"])
@pytest.mark.parametrize("B,T", [(1, 700), (5, 256)])
def test_noalloc_matches_workspace_entry_on_two_calls_in_a_row(B, T, flags):
    from tests.helpers import assert_bit_exact
    from tests.test_gpu_mixer import make_layer, mixer_inputs
    shape = W.SHAPE_QWEN
    m, _ = make_layer(shape, "bf16", seed=21)
    dev = torch.device("cuda")
    if B * shape.num_v_heads > 148:
        assert torch.cuda.get_device_properties(dev).multi_processor_count < B * shape.num_v_heads
    lib = _lib.load()
    t = lambda a: torch.from_numpy(a).to(dev).to(torch.bfloat16)  # noqa: E731
    for call in range(2):
        d = mixer_inputs(shape, B, T, "bf16", seed=200 + 10 * B + call, with_state=True)
        ins = (t(d["mixed"]), t(d["z"]), t(d["b"]), t(d["a"]))
        cs_in, S_in = t(d["conv_state"]), torch.from_numpy(d["rec_state"]).to(dev)
        results = []
        for entry in ("ws", "noalloc"):
            out = torch.full((B, T, shape.value_dim), float("nan"), dtype=torch.bfloat16, device=dev)
            S = torch.full_like(S_in, float("nan"))
            cs = torch.zeros_like(cs_in)
            args, out, keep = m._mixer_args(*ins, cs_in, S_in, cs, S, out, flags)
            nbytes = lib.gdn_prefill_workspace_bytes(ctypes.byref(args))
            assert 0 <= nbytes <= _lib.GDN_STATIC_SCRATCH_BYTES
            if B * shape.num_v_heads > 148:  # state hand-offs between CTAs: their flags live in the scratch
                assert nbytes > 0
            stream = torch.cuda.current_stream(dev).cuda_stream
            if entry == "ws":
                ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
                _lib.check("gdn_mixer_prefill_ws",
                           lib.gdn_mixer_prefill_ws(ctypes.byref(args), ws.data_ptr() if nbytes else None, nbytes,
                                                    stream))
            else:
                _lib.check("gdn_mixer_prefill_noalloc", lib.gdn_mixer_prefill_noalloc(ctypes.byref(args), stream))
            torch.cuda.synchronize()
            results.append((out.float().cpu().numpy(), S.cpu().numpy(), cs.float().cpu().numpy()))
        for (name, a), (_, b) in zip((("out", results[0][0]), ("state", results[0][1]), ("conv", results[0][2])),
                                     (("out", results[1][0]), ("state", results[1][1]), ("conv", results[1][2]))):
            assert np.isfinite(a).all(), name
            assert_bit_exact(b, a, f"call {call} {name}")
    assert _lib.device_error() == 0
