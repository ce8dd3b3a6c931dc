"""Speculative-decode verify with per-row state slots (gdn_mixer_verify_slots +
gdn_accept_slots): parity with the oracle's rollback semantics, bit-exactness
against the checkpoint-and-copy path at the rollback workload's full size
(B16, 16/32 heads, d128, 4-token drafts, 1024 steps), slot-table index parity,
and the kernels' own range checks."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gdn_oracle as O
from tests.helpers import assert_bf16_close, assert_bit_exact, assert_state_close
from tests.test_gpu_mixer import make_layer, mixer_inputs
from visionstack_b200 import StateSlots, _lib
from visionstack_b200 import workloads as W

pytestmark = pytest.mark.gpu


def simulate_table(batch: int, num_slots: int, accepted_steps) -> np.ndarray:
    """Host model of the slot table: accepting a tokens swaps columns 0 and a."""
    table = np.tile(np.arange(num_slots, dtype=np.int32), (batch, 1))
    for acc in accepted_steps:
        for row, a in enumerate(acc):
            if a:
                table[row, 0], table[row, a] = table[row, a], table[row, 0]
    return table


def _t(a, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda().to(dtype)


def test_verify_slots_matches_oracle_rollback():
    shape = W.LayerShape(256, 2, 4, 128, 128)
    m, params = make_layer(shape, "bf16", seed=4)
    B, T, steps = 3, 4, 6
    d0 = mixer_inputs(shape, B, T, "bf16", seed=90, with_state=True)
    conv, rec = d0["conv_state"], d0["rec_state"]
    slots = StateSlots(m, B, T, torch.bfloat16, torch.device("cuda"))
    slots.load(_t(conv), torch.from_numpy(rec).cuda())
    accepts = np.array([[0, 4, 2], [1, 0, 4], [3, 3, 0], [4, 1, 1], [0, 0, 0], [2, 4, 3]], dtype=np.int32)
    for step in range(steps):
        d = mixer_inputs(shape, B, T, "bf16", seed=100 + step, with_state=False)
        out = m.mixer_verify(_t(d["mixed"]), _t(d["z"]), _t(d["b"]), _t(d["a"]), slots)
        for t in range(T + 1):
            cs_t, _ = slots.after(t)
            if t == 0:
                assert_bit_exact(cs_t, conv, f"step {step} starting conv state")
        slots.accept(torch.from_numpy(accepts[step]).cuda())
        r_out, conv, rec = O.speculative_verify_rollback(
            shape, d["mixed"], d["z"].reshape(B, T, shape.num_v_heads, shape.head_v_dim), d["a"], d["b"],
            params["conv1d.weight"], params["A_log"], params["dt_bias"], params["norm.weight"], "bf16", conv, rec,
            accepts[step])
        assert_bf16_close(out, r_out, f"step {step} out")
        c_cur, r_cur = slots.current()
        assert_bit_exact(c_cur, conv, f"step {step} conv state")
        assert_state_close(r_cur, rec, f"step {step} state")
    assert_bit_exact(slots.table.cpu().numpy(), simulate_table(B, T + 1, accepts), "slot table")
    assert _lib.device_error() == 0


def test_verify_slots_bit_exact_against_checkpoint_copy_path_full_size():
    """The rollback workload at full size: every step's output and the final
    states equal, bit for bit, those of the reference-shaped path (token-by-
    token mixer with checkpoints after every token into separate buffers, then a
    per-row copy of the accepted checkpoint, the pre-draft state kept for 0)."""
    wl = W.WORKLOADS["rollback"]
    shape, B, T, steps = wl.shape, wl.batch, wl.seq_len, wl.steps
    m, _ = make_layer(shape, "bf16", seed=5)
    gen = torch.Generator(device="cuda").manual_seed(55)
    dev = torch.device("cuda")
    conv0 = (0.7 * torch.randn((B, shape.conv_dim, 3), device=dev, generator=gen)).bfloat16()
    rec0 = 0.02 * torch.randn((B, shape.num_v_heads, 128, 128), device=dev, generator=gen)
    accepts = torch.from_numpy(np.random.default_rng(wl.x_seed).integers(0, T + 1, size=(steps, B))).to(dev)
    n_in = 8  # distinct input sets, reused round-robin
    ins = [tuple((0.7 * torch.randn(s, device=dev, generator=gen)).bfloat16()
                 for s in ((B, T, shape.conv_dim), (B, T, shape.value_dim), (B, T, shape.num_v_heads),
                           (B, T, shape.num_v_heads))) for _ in range(n_in)]

    slots = StateSlots(m, B, T, torch.bfloat16, dev)
    slots.load(conv0, rec0)
    conv, rec = conv0.clone(), rec0.clone()
    rows = torch.arange(B, device=dev)
    st_ck = torch.empty((T + 1, B, shape.num_v_heads, 128, 128), device=dev)
    cv_ck = torch.empty((T + 1, B, shape.conv_dim, 3), dtype=torch.bfloat16, device=dev)
    with torch.inference_mode():
        for step in range(steps):
            mixed, z, b, a = ins[step % n_in]
            out_s = m.mixer_verify(mixed, z, b, a, slots)
            slots.accept(accepts[step])
            st_ck[0].copy_(rec)
            cv_ck[0].copy_(conv)
            out_r = m.mixer(mixed, z, b, a, conv_state=conv, rec_state=rec, conv_state_out=None,
                            rec_state_out=None, checkpoint_offsets=list(range(1, T + 1)),
                            state_checkpoints=st_ck[1:], conv_checkpoints=cv_ck[1:], token_by_token=True)
            acc = accepts[step]
            rec = st_ck[acc, rows].clone()
            conv = cv_ck[acc, rows].clone()
            if step % 128 == 0 or step == steps - 1:
                assert torch.equal(out_s, out_r), f"step {step}: outputs differ"
    torch.cuda.synchronize()
    c_cur, r_cur = slots.current()
    assert torch.equal(c_cur, conv), "conv states differ"
    assert torch.equal(r_cur, rec), "recurrent states differ"
    assert_bit_exact(slots.table.cpu().numpy(), simulate_table(B, T + 1, accepts.cpu().numpy()), "slot table")
    assert _lib.device_error() == 0


def test_layer_verify_equals_forward_with_checkpoints():
    """Qwen3_5GatedDeltaNet.verify on slots gives the forward's output, and
    after accepting a tokens the slots hold the cache checkpoint at a."""
    from visionstack_b200 import Qwen3_5HybridCache
    shape = W.LayerShape(512, 4, 8, 128, 128)
    m, _ = make_layer(shape, "bf16", seed=6)
    B, T = 4, 4
    gen = torch.Generator(device="cuda").manual_seed(7)
    x0 = torch.randn((B, 20, shape.hidden_size), device="cuda", generator=gen).bfloat16()
    xd = torch.randn((B, T, shape.hidden_size), device="cuda", generator=gen).bfloat16()
    with torch.inference_mode():
        cache = Qwen3_5HybridCache()
        m(x0, cache=cache)
        cache.past_seen_tokens = 20
        slots = StateSlots(m, B, T, torch.bfloat16, torch.device("cuda"))
        slots.load(cache.conv_states[0], cache.recurrent_states[0])
        y_s = m.verify(xd, slots)
        ver = cache.clone_and_expand(1, record_checkpoints=True, checkpoint_positions=list(range(21, 21 + T)))
        ver.resolve_active_checkpoints(20, T)
        y_r = m(xd, cache=ver)
        slots.accept(torch.tensor([0, 1, 2, 4], device="cuda"))
    torch.cuda.synchronize()
    assert torch.equal(y_s, y_r)
    c_cur, r_cur = slots.current()
    for row, acc in enumerate([0, 1, 2, 4]):
        if acc == 0:
            rc, rr = cache.conv_states[0][row], cache.recurrent_states[0][row]
        else:
            rc, rr = ver.conv_checkpoints[20 + acc][0][row], ver.recurrent_checkpoints[20 + acc][0][row]
        assert torch.equal(c_cur[row], rc), f"row {row} conv"
        assert torch.equal(r_cur[row], rr), f"row {row} state"


def test_out_of_range_slots_and_counts_are_flagged_not_followed():
    """A slot-table entry or an accepted count out of range is caught by the
    kernels' own range checks: nothing outside the pools is touched, the row's
    table is unchanged, and the device error word reports it."""
    shape = W.LayerShape(256, 2, 4, 128, 128)
    m, _ = make_layer(shape, "bf16", seed=8)
    B, T = 2, 4
    slots = StateSlots(m, B, T, torch.bfloat16, torch.device("cuda"))
    d = mixer_inputs(shape, B, T, "bf16", seed=120, with_state=False)
    _lib.device_error(clear=True)
    slots.table[1, 3] = 99  # row 1's slot for token 3 is out of range
    before = slots.state.clone()
    m.mixer_verify(_t(d["mixed"]), _t(d["z"]), _t(d["b"]), _t(d["a"]), slots)
    torch.cuda.synchronize()
    assert _lib.device_error(clear=True) & _lib.GDN_DEVERR_BAD_SLOT
    assert torch.equal(slots.state[3, 1], before[3, 1]), "slot 3 of row 1 was written through a bad entry"
    slots.table[1, 3] = 3
    m.mixer_verify(_t(d["mixed"]), _t(d["z"]), _t(d["b"]), _t(d["a"]), slots)
    table = slots.table.clone()
    slots.accept(torch.tensor([7, -1], device="cuda", dtype=torch.int32))
    torch.cuda.synchronize()
    assert _lib.device_error(clear=True) & _lib.GDN_DEVERR_BAD_SLOT
    assert torch.equal(slots.table, table)
    assert _lib.device_error() == 0
