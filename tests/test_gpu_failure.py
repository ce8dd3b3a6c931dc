"""Failure detection on the GPU without a fault: every spin-wait in the pipelined kernels is
bounded, records a device error bit when it gives up and returns.  Here the wait is made to run
out on purpose (an mbarrier nothing arrives at, a hand-off flag nothing sets); the test checks
the recorded status, that the kernel returned after about the limit, and that the context still
runs the mixer correctly afterwards.
"""
from __future__ import annotations

import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def _expired_wait(kind: int, preset: int = 0):
    from visionstack_b200 import _lib
    lib = _lib.load()
    flag = torch.zeros(2, dtype=torch.int32, device="cuda")
    flag[0] = preset
    _lib.device_error(clear=True)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    _lib.check("gdn_selftest_expired_wait", lib.gdn_selftest_expired_wait(kind, flag.data_ptr(), None))
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    return int(flag[1].item()), _lib.device_error(clear=True), dt


@pytest.mark.parametrize("kind,bit", [(0, 0x1), (1, 0x8)], ids=["mbarrier", "handoff_flag"])
def test_wait_that_never_completes_gives_up_and_reports(kind, bit):
    result, err, dt = _expired_wait(kind)
    assert result == 2, "the wait should have given up"
    assert err == bit
    assert 0.9 < dt < 30.0


def test_flag_already_set_passes_without_error():
    result, err, dt = _expired_wait(1, preset=1)
    assert result == 1 and err == 0
    assert dt < 0.9


def test_context_usable_after_an_expired_wait():
    from tests.test_gpu_mixer import check, make_layer, mixer_inputs, run_oracle, run_ours
    from visionstack_b200 import _lib
    from visionstack_b200 import workloads as W
    result, err, _ = _expired_wait(1)
    assert result == 2 and err == 0x8
    shape = W.SHAPE_SMALL
    m, params = make_layer(shape, "bf16")
    d = mixer_inputs(shape, 2, 130, "bf16", seed=41, with_state=True)
    ours = run_ours(m, shape, d, "bf16", False, (64, 130))
    assert _lib.device_error(clear=True) == 0
    check(shape, "bf16", ours, run_oracle(shape, params, d, "bf16", chunk=True, offsets=(64, 130)), (64, 130),
          "after an expired wait")


def test_peer_allreduce_wait_runs_out_and_context_survives():
    """A one-shot peer all-reduce whose other rank never arrives: the "peer" here is a second
    staging allocation on the same GPU that nothing writes, so the wait for its flag runs out
    after the 1 s limit, the kernel sets GDN_DEVERR_PEER_TIMEOUT and returns; the context then
    runs an all-reduce of a group of one."""
    import ctypes
    import time

    from visionstack_b200 import _lib
    lib = _lib.load()
    cap, nb = 1024, 1
    nbytes = lib.gdn_peer_staging_bytes(2, nb, cap)
    mine, other = ctypes.c_void_p(), ctypes.c_void_p()
    _lib.check("alloc", lib.gdn_peer_staging_alloc(nbytes, ctypes.byref(mine)))
    _lib.check("alloc", lib.gdn_peer_staging_alloc(nbytes, ctypes.byref(other)))
    try:
        _lib.device_error(clear=True)
        g = _lib.PeerGroup()
        g.rank, g.world, g.nblocks, g.cap = 0, 2, nb, cap
        g.staging[0], g.staging[1] = mine.value, other.value
        x = torch.ones(cap, dtype=torch.bfloat16, device="cuda")
        y = torch.zeros_like(x)
        t0 = time.monotonic()
        _lib.check("peer", lib.gdn_peer_allreduce_bf16(ctypes.byref(g), x.data_ptr(), y.data_ptr(), cap, None))
        torch.cuda.synchronize()
        dt = time.monotonic() - t0
        assert _lib.device_error(clear=True) & _lib.GDN_DEVERR_PEER_TIMEOUT
        assert 0.9 < dt < 30.0, dt
        assert float(y.float().abs().max()) == 0.0  # the block gave up before writing the output
        # a group of one on fresh staging memory: the sum is the input itself
        g1 = _lib.PeerGroup()
        g1.rank, g1.world, g1.nblocks, g1.cap = 0, 1, nb, cap
        g1.staging[0] = other.value
        _lib.check("peer", lib.gdn_peer_allreduce_bf16(ctypes.byref(g1), x.data_ptr(), y.data_ptr(), cap, None))
        torch.cuda.synchronize()
        assert torch.equal(y, x) and _lib.device_error() == 0
    finally:
        torch.cuda.synchronize()
        lib.gdn_peer_staging_free(mine)
        lib.gdn_peer_staging_free(other)
