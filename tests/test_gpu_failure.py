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
