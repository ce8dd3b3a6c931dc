"""CPU oracle: a numpy restatement of the reference Gated DeltaNet token mixer.

TEST INFRASTRUCTURE, NOT PRODUCT CODE.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its CPU-baseline leg and its
``--impl reference`` arm) may import this module, and only as the checker or as
the timed CPU baseline.  The product path (``visionstack_b200``) never imports
it and has no CPU fallback.

Every function restates the algorithm of the reference file
``ShadowBoxer/models/qwen35/deltanet.py`` (and the helpers it uses from
``ShadowBoxer/models/qwen35/config.py``) at the cited lines.  Arithmetic is
float32 (numpy single precision) and "bf16" tensors are float32 arrays whose
values have been rounded to bfloat16 after every operation that the reference
performs in bfloat16, so that the rounding points match the reference's
PyTorch ops.

Parity pin: this oracle is checked against fixtures produced by running the
reference itself (``tests/golden/make_golden.py``), see
``tests/test_oracle_golden.py``.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

from visionstack_b200.workloads import cast, round_bf16  # noqa: F401  (numpy-only helpers)

F32 = np.float32


def silu(x: np.ndarray) -> np.ndarray:
    x = x.astype(F32, copy=False)
    return (x / (F32(1.0) + np.exp(-x))).astype(F32)


def sigmoid(x: np.ndarray) -> np.ndarray:
    x = x.astype(F32, copy=False)
    return (F32(1.0) / (F32(1.0) + np.exp(-x))).astype(F32)


def softplus(x: np.ndarray) -> np.ndarray:
    """torch.nn.functional.softplus with beta=1, threshold=20."""
    x = x.astype(F32, copy=False)
    with np.errstate(over="ignore"):
        y = np.log1p(np.exp(x)).astype(F32)
    return np.where(x > F32(20.0), x, y).astype(F32)


# ---------------------------------------------------------------------------
# Convolution (deltanet.py:24-90)
# ---------------------------------------------------------------------------

def extract_conv_state_at_offset(x: np.ndarray, prev_state: Optional[np.ndarray],
                                 local_offset: int, state_len: int = 3) -> np.ndarray:
    """Raw (pre-conv) inputs of positions [off-state_len, off), deltanet.py:24-38.

    ``x`` is [B, C, T]; positions before 0 come from ``prev_state`` (oldest
    first) or are zero when there is no previous state.
    """
    if local_offset >= state_len:
        return np.ascontiguousarray(x[:, :, local_offset - state_len:local_offset])
    if prev_state is not None:
        return np.ascontiguousarray(
            np.concatenate([prev_state[:, :, local_offset:], x[:, :, :local_offset]], axis=-1))
    pad = state_len - local_offset
    out = np.zeros(x.shape[:2] + (state_len,), dtype=x.dtype)
    out[:, :, pad:] = x[:, :, :local_offset]
    return out


def causal_conv1d(x: np.ndarray, weight: np.ndarray, conv_state: Optional[np.ndarray] = None,
                  activation: Optional[str] = "silu", return_final_state: bool = False,
                  w_dtype: str = "f32", act_dtype: str = "f32"):
    """Depthwise causal conv + activation, deltanet.py:41-90.

    ``x`` [B, C, T] in ``act_dtype``; ``weight`` [C, K] in ``w_dtype``.  The
    reference computes in the weight dtype: the newest tap first
    (``x * w[:, K-1]``), then the in-sequence taps (``addcmul_``, one rounding
    per tap), then the taps that reach into ``conv_state``.
    """
    B, C, T = x.shape
    w = weight.reshape(C, -1).astype(F32)
    K = w.shape[-1]
    L = K - 1
    new_state = extract_conv_state_at_offset(x, conv_state, T, L) if return_final_state else None
    xt = cast(x, w_dtype)
    out = cast(xt * w[:, K - 1][None, :, None], w_dtype)
    for tap in range(1, min(K, T)):
        out[:, :, tap:] = cast(out[:, :, tap:] + xt[:, :, :-tap] * w[:, K - 1 - tap][None, :, None], w_dtype)
    if conv_state is not None and L > 0:
        cs = cast(conv_state, w_dtype)
        for tap in range(1, K):
            n = min(tap, T)
            s0 = L - tap
            out[:, :, :n] = cast(out[:, :, :n] + cs[:, :, s0:s0 + n] * w[:, K - 1 - tap][None, :, None], w_dtype)
    if activation:
        out = cast(silu(out), w_dtype)
    res = cast(out, act_dtype)
    if return_final_state:
        return res, new_state
    return res


# ---------------------------------------------------------------------------
# Delta rule (deltanet.py:93-407, config.py:114-115)
# ---------------------------------------------------------------------------

def l2norm(x: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """x * rsqrt(sum(x^2) + eps) over the last axis, config.py:114-115."""
    x = x.astype(F32, copy=False)
    ss = np.sum(x * x, axis=-1, keepdims=True, dtype=F32)
    return (x * (F32(1.0) / np.sqrt(ss + F32(eps)))).astype(F32)


def invert_unit_lower_triangular_block(u: np.ndarray) -> np.ndarray:
    """(I + tril(u, -1))^-1 by Neumann-series products, deltanet.py:93-109."""
    n = u.shape[-1]
    eye = np.eye(n, dtype=F32)
    a = -np.tril(u, -1).astype(F32)
    inv = eye + a
    if n == 16:
        a2 = a @ a
        a4 = a2 @ a2
        a8 = a4 @ a4
        return (((inv @ (eye + a2)) @ (eye + a4)) @ (eye + a8)).astype(F32)
    cur = a
    step = 1
    while step < n:
        cur = cur @ cur
        inv = inv @ (eye + cur)
        step <<= 1
    return inv.astype(F32)


def solve_unit_lower_triangular(ut: np.ndarray, rhs: np.ndarray) -> np.ndarray:
    """(I + tril(ut, -1))^-1 @ rhs: 16x16 diagonal-block inverses merged by
    2x2 block doubling (T21 = -T22 U21 T11), deltanet.py:112-162."""
    n = ut.shape[-1]
    if n <= 16 or (n & (n - 1)) != 0:
        return (invert_unit_lower_triangular_block(ut) @ rhs).astype(F32)
    bs = 16
    nb = n // bs
    batch = ut.shape[:-2]
    blocks = ut.reshape(*batch, nb, bs, nb, bs)
    diag = np.stack([blocks[..., i, :, i, :] for i in range(nb)], axis=-3)
    inv = invert_unit_lower_triangular_block(diag)  # [..., nb, bs, bs]
    cur, num = bs, nb
    while num > 1:
        half = num // 2
        inv_r = inv.reshape(*batch, half, 2, cur, cur)
        t11 = inv_r[..., 0, :, :]
        t22 = inv_r[..., 1, :, :]
        part = ut.reshape(*batch, half, 2, cur, half, 2, cur)
        u21 = np.stack([part[..., p, 1, :, p, 0, :] for p in range(half)], axis=-3)
        t21 = -(t22 @ (u21 @ t11))
        nxt = np.zeros((*batch, half, 2 * cur, 2 * cur), dtype=F32)
        nxt[..., :cur, :cur] = t11
        nxt[..., cur:, :cur] = t21
        nxt[..., cur:, cur:] = t22
        inv = nxt
        cur *= 2
        num = half
    return (inv[..., 0, :, :] @ rhs).astype(F32)


def recurrent_gated_delta_rule(q, k, v, g, beta, initial_state=None, output_final_state=False,
                               use_qk_l2norm=True, checkpoint_positions: Optional[Sequence[int]] = None,
                               checkpoint_states_out: Optional[Dict[int, np.ndarray]] = None,
                               past_seen_tokens: int = 0, out_dtype: str = "f32"):
    """Token-by-token delta rule, deltanet.py:165-233.

    q, k [B, T, H, dk]; v [B, T, H, dv]; g, beta [B, T, H].  Per token:
    S <- S * exp(g); u = beta (v - k S); S <- S + k^T u; o = q S.
    """
    B, T, H, dk = k.shape
    dv = v.shape[-1]
    qf = np.ascontiguousarray(np.transpose(q, (0, 2, 1, 3))).astype(F32)
    kf = np.ascontiguousarray(np.transpose(k, (0, 2, 1, 3))).astype(F32)
    vf = np.ascontiguousarray(np.transpose(v, (0, 2, 1, 3))).astype(F32)
    bf = np.ascontiguousarray(np.transpose(beta, (0, 2, 1))).astype(F32)
    gf = np.ascontiguousarray(np.transpose(g, (0, 2, 1))).astype(F32)
    if use_qk_l2norm:
        qf = l2norm(qf)
        kf = l2norm(kf)
    qf = (qf * F32(dk ** -0.5)).astype(F32)
    decay = np.exp(gf).astype(F32)
    S = (np.array(initial_state, dtype=F32, copy=True) if initial_state is not None
         else np.zeros((B, H, dk, dv), dtype=F32))
    out = np.empty((B, H, T, dv), dtype=F32)
    cps = set(int(c) for c in checkpoint_positions) if checkpoint_positions else None
    for t in range(T):
        S = S * decay[:, :, t][:, :, None, None]
        kt = kf[:, :, t, :]
        v_pred = np.matmul(kt[:, :, None, :], S)[:, :, 0, :]
        u = bf[:, :, t][:, :, None] * (vf[:, :, t, :] - v_pred)
        S = S + kt[:, :, :, None] * u[:, :, None, :]
        out[:, :, t, :] = np.matmul(qf[:, :, t, :][:, :, None, :], S)[:, :, 0, :]
        if cps is not None and checkpoint_states_out is not None:
            pos = past_seen_tokens + t + 1
            if pos in cps:
                checkpoint_states_out[pos] = S.copy()
    o = cast(np.ascontiguousarray(np.transpose(out, (0, 2, 1, 3))), out_dtype)
    if output_final_state:
        return o, S
    return o


def chunk_gated_delta_rule(q, k, v, g, beta, chunk_size: int = 64, initial_state=None,
                           output_final_state=False, use_qk_l2norm=True,
                           checkpoint_positions: Optional[Sequence[int]] = None,
                           checkpoint_states_out: Optional[Dict[int, np.ndarray]] = None,
                           past_seen_tokens: int = 0, out_dtype: str = "f32"):
    """Chunked WY/UT form of the delta rule, deltanet.py:236-407.

    Dispatch rules of the reference: with an initial state and T <= 8 the
    token-by-token form runs (deltanet.py:251-264); chunk 64 shrinks to 16 for
    T <= 16 and to 32 for T <= 32 (deltanet.py:272-276).
    """
    T = k.shape[1]
    if initial_state is not None and T <= 8:
        return recurrent_gated_delta_rule(q, k, v, g, beta, initial_state, output_final_state,
                                          use_qk_l2norm, checkpoint_positions,
                                          checkpoint_states_out, past_seen_tokens, out_dtype)
    B, _, H, dk = k.shape
    dv = v.shape[-1]
    C = chunk_size
    if C == 64:
        if T <= 16:
            C = 16
        elif T <= 32:
            C = 32
    qf = np.ascontiguousarray(np.transpose(q, (0, 2, 1, 3))).astype(F32)
    kf = np.ascontiguousarray(np.transpose(k, (0, 2, 1, 3))).astype(F32)
    vf = np.ascontiguousarray(np.transpose(v, (0, 2, 1, 3))).astype(F32)
    bf = np.ascontiguousarray(np.transpose(beta, (0, 2, 1))).astype(F32)
    gf = np.ascontiguousarray(np.transpose(g, (0, 2, 1))).astype(F32)
    if use_qk_l2norm:
        qf = l2norm(qf)
        kf = l2norm(kf)
    qf = (qf * F32(dk ** -0.5)).astype(F32)
    pad = (C - T % C) % C
    if pad:
        qf = np.pad(qf, ((0, 0), (0, 0), (0, pad), (0, 0)))
        kf = np.pad(kf, ((0, 0), (0, 0), (0, pad), (0, 0)))
        vf = np.pad(vf, ((0, 0), (0, 0), (0, pad), (0, 0)))
        bf = np.pad(bf, ((0, 0), (0, 0), (0, pad)))
        gf = np.pad(gf, ((0, 0), (0, 0), (0, pad)))
    NC = (T + pad) // C
    v_beta = vf * bf[..., None]
    k_beta = kf * bf[..., None]
    qc = qf.reshape(B, H, NC, C, dk)
    kc = kf.reshape(B, H, NC, C, dk)
    kbc = k_beta.reshape(B, H, NC, C, dk)
    vbc = v_beta.reshape(B, H, NC, C, dv)
    gamma = np.cumsum(gf.reshape(B, H, NC, C), axis=-1, dtype=F32)
    e_gamma = np.exp(gamma).astype(F32)
    upper = np.triu(np.ones((C, C), dtype=bool), 1)
    with np.errstate(over="ignore"):
        pair = np.exp(gamma[..., :, None] - gamma[..., None, :]).astype(F32)
    pair = np.where(upper, F32(0.0), pair).astype(F32)
    kT = np.swapaxes(kc, -1, -2)
    ut = (kbc @ kT) * pair
    intra = (qc @ kT) * pair
    rhs = np.concatenate([vbc, kbc * e_gamma[..., None]], axis=-1)
    solved = solve_unit_lower_triangular(ut.astype(F32), rhs.astype(F32))
    new_values = solved[..., :dv]
    k_cumdecay = solved[..., dv:]
    S = (np.array(initial_state, dtype=F32, copy=True) if initial_state is not None
         else np.zeros((B, H, dk, dv), dtype=F32))
    out = np.zeros((B, H, NC, C, dv), dtype=F32)

    cp_map: Dict[int, List[Tuple[int, int]]] = {}
    if checkpoint_positions and checkpoint_states_out is not None:
        for cp in checkpoint_positions:
            local = int(cp) - past_seen_tokens
            if 1 <= local <= T:
                ci = (local - 1) // C
                cp_map.setdefault(ci, []).append((local - ci * C, int(cp)))

    q_dec = qc * e_gamma[..., None]
    k_dec = kc * np.exp(gamma[..., -1:] - gamma)[..., None]
    chunk_decay = e_gamma[..., -1][..., None, None]
    for i in range(NC):
        v_new = new_values[:, :, i] - k_cumdecay[:, :, i] @ S
        out[:, :, i] = q_dec[:, :, i] @ S + intra[:, :, i] @ v_new
        S_next = S * chunk_decay[:, :, i] + np.swapaxes(k_dec[:, :, i], -1, -2) @ v_new
        for s_off, abs_cp in cp_map.get(i, []):
            if s_off == C:
                checkpoint_states_out[abs_cp] = S_next.copy()
            else:
                dec_s = gamma[:, :, i, s_off - 1:s_off]
                k_s = kc[:, :, i, :s_off] * np.exp(dec_s - gamma[:, :, i, :s_off])[..., None]
                checkpoint_states_out[abs_cp] = (
                    S * np.exp(dec_s)[..., None] + np.swapaxes(k_s, -1, -2) @ v_new[:, :, :s_off]
                ).astype(F32)
        S = S_next.astype(F32)
    o = out.reshape(B, H, -1, dv)[:, :, :T]
    o = cast(np.ascontiguousarray(np.transpose(o, (0, 2, 1, 3))), out_dtype)
    if output_final_state:
        return o, S
    return o


# ---------------------------------------------------------------------------
# Gated RMSNorm (config.py:130-143) and the layer (deltanet.py:410-563)
# ---------------------------------------------------------------------------

def rms_norm_gated(h: np.ndarray, gate: np.ndarray, weight: np.ndarray, eps: float, dtype: str) -> np.ndarray:
    """RMS over the last axis, rounded to the input dtype, times weight (in the
    input dtype), times SiLU(gate) in fp32, config.py:136-143."""
    hf = h.astype(F32)
    var = np.mean(hf * hf, axis=-1, keepdims=True, dtype=F32)
    normed = hf * (F32(1.0) / np.sqrt(var + F32(eps)))
    scaled = cast(weight.astype(F32) * cast(normed, dtype), dtype)
    return cast(scaled * silu(gate.astype(F32)), dtype)


class OracleCache:
    """The fields of the reference's hybrid cache that the layer touches
    (ShadowBoxer/models/qwen35/cache.py:9-37)."""

    def __init__(self, record_checkpoints: bool = False, checkpoint_offsets: Sequence[int] = ()):
        self.conv_states: Dict[int, np.ndarray] = {}
        self.recurrent_states: Dict[int, np.ndarray] = {}
        self.past_seen_tokens = 0
        self.record_checkpoints = bool(record_checkpoints)
        self.checkpoint_offsets: List[int] = list(checkpoint_offsets)
        self.conv_checkpoints: Dict[int, Dict[int, np.ndarray]] = {}
        self.recurrent_checkpoints: Dict[int, Dict[int, np.ndarray]] = {}


def linear(x: np.ndarray, w: np.ndarray, dtype: str) -> np.ndarray:
    return cast(np.matmul(x.astype(F32), w.astype(F32).T), dtype)


def deltanet_layer_forward(params: Dict[str, np.ndarray], shape, x: np.ndarray, dtype: str,
                           attention_mask: Optional[np.ndarray] = None,
                           cache: Optional[OracleCache] = None, layer_idx: int = 0) -> np.ndarray:
    """One Gated DeltaNet layer with the reference's cache side effects,
    deltanet.py:447-563.  ``params`` uses the reference state-dict names."""
    if attention_mask is not None and attention_mask.ndim == 2:
        x = cast(x * attention_mask[:, :, None].astype(F32), dtype)
    B, T, _ = x.shape
    Hk, Hv, dk, dv = shape.num_k_heads, shape.num_v_heads, shape.head_k_dim, shape.head_v_dim
    mixed = np.ascontiguousarray(np.transpose(linear(x, params["in_proj_qkv.weight"], dtype), (0, 2, 1)))
    z = linear(x, params["in_proj_z.weight"], dtype).reshape(B, T, Hv, dv)
    b = linear(x, params["in_proj_b.weight"], dtype)
    a = linear(x, params["in_proj_a.weight"], dtype)
    prev_conv = cache.conv_states.get(layer_idx) if cache is not None else None
    prev_rec = cache.recurrent_states.get(layer_idx) if cache is not None else None
    past = cache.past_seen_tokens if cache is not None else 0
    cps = cache.checkpoint_offsets if (cache is not None and cache.record_checkpoints) else None
    L = shape.conv_kernel - 1
    if cps and cache is not None:
        for cp in cps:
            off = cp - past
            if 1 <= off <= T:
                cache.conv_checkpoints.setdefault(cp, {})[layer_idx] = extract_conv_state_at_offset(
                    mixed, prev_conv, off, L)
    w = params["conv1d.weight"].reshape(shape.conv_dim, -1)
    if cache is not None:
        conv_out, nxt = causal_conv1d(mixed, w, prev_conv, "silu", True, dtype, dtype)
        cache.conv_states[layer_idx] = nxt
    else:
        conv_out = causal_conv1d(mixed, w, None, "silu", False, dtype, dtype)
    mq = np.transpose(conv_out, (0, 2, 1))
    kd = Hk * dk
    q = mq[..., :kd].reshape(B, T, Hk, dk)
    k = mq[..., kd:2 * kd].reshape(B, T, Hk, dk)
    v = mq[..., 2 * kd:].reshape(B, T, Hv, dv)
    beta = cast(sigmoid(b), dtype)
    g = (-np.exp(params["A_log"].astype(F32)) * softplus(a.astype(F32) + params["dt_bias"].astype(F32))).astype(F32)
    rep = Hv // Hk
    if rep > 1:
        q = np.repeat(q, rep, axis=2)
        k = np.repeat(k, rep, axis=2)
    if cache is not None:
        rec_cps: Optional[Dict[int, np.ndarray]] = {} if cps else None
        o, S = chunk_gated_delta_rule(q, k, v, g, beta, initial_state=prev_rec, output_final_state=True,
                                      checkpoint_positions=cps, checkpoint_states_out=rec_cps,
                                      past_seen_tokens=past, out_dtype=dtype)
        cache.recurrent_states[layer_idx] = S
        if rec_cps:
            for cp, st in rec_cps.items():
                cache.recurrent_checkpoints.setdefault(cp, {})[layer_idx] = st
    else:
        o = chunk_gated_delta_rule(q, k, v, g, beta, out_dtype=dtype)
    normed = rms_norm_gated(o.reshape(-1, dv), z.reshape(-1, dv), params["norm.weight"],
                            shape.rms_norm_eps, dtype).reshape(B, T, -1)
    return linear(normed, params["out_proj.weight"], dtype)


def mixer_forward(shape, mixed_qkv: np.ndarray, z: np.ndarray, a: np.ndarray, b: np.ndarray,
                  conv_w: np.ndarray, A_log: np.ndarray, dt_bias: np.ndarray, norm_w: np.ndarray,
                  dtype: str, conv_state: Optional[np.ndarray] = None,
                  rec_state: Optional[np.ndarray] = None, chunk: bool = True,
                  checkpoint_offsets: Sequence[int] = ()):
    """The token mixer between the input projections and out_proj
    (deltanet.py:479-561) on projection outputs: mixed_qkv [B, T, conv_dim],
    z [B, T, Hv, dv], a/b [B, T, Hv].  Returns (gated-norm output [B, T, Hv*dv],
    new conv state, new recurrent state, {offset: conv checkpoint},
    {offset: recurrent checkpoint}) with checkpoint offsets local (1..T)."""
    B, T, _ = mixed_qkv.shape
    Hk, Hv, dk, dv = shape.num_k_heads, shape.num_v_heads, shape.head_k_dim, shape.head_v_dim
    mixed = np.ascontiguousarray(np.transpose(mixed_qkv, (0, 2, 1)))
    L = shape.conv_kernel - 1
    conv_cps = {off: extract_conv_state_at_offset(mixed, conv_state, off, L)
                for off in checkpoint_offsets if 1 <= off <= T}
    conv_out, nxt = causal_conv1d(mixed, conv_w.reshape(shape.conv_dim, -1), conv_state, "silu", True,
                                  dtype, dtype)
    mq = np.transpose(conv_out, (0, 2, 1))
    kd = Hk * dk
    q = mq[..., :kd].reshape(B, T, Hk, dk)
    k = mq[..., kd:2 * kd].reshape(B, T, Hk, dk)
    v = mq[..., 2 * kd:].reshape(B, T, Hv, dv)
    beta = cast(sigmoid(b), dtype)
    g = (-np.exp(A_log.astype(F32)) * softplus(a.astype(F32) + dt_bias.astype(F32))).astype(F32)
    rep = Hv // Hk
    if rep > 1:
        q = np.repeat(q, rep, axis=2)
        k = np.repeat(k, rep, axis=2)
    fn = chunk_gated_delta_rule if chunk else recurrent_gated_delta_rule
    rec_cps: Dict[int, np.ndarray] = {}
    o, S = fn(q, k, v, g, beta, initial_state=rec_state, output_final_state=True, out_dtype=dtype,
              checkpoint_positions=list(checkpoint_offsets) or None, checkpoint_states_out=rec_cps)
    out = rms_norm_gated(o.reshape(-1, dv), z.reshape(-1, dv), norm_w, shape.rms_norm_eps, dtype)
    return out.reshape(B, T, Hv * dv), nxt, S, conv_cps, rec_cps


def speculative_verify_rollback(shape, mixed_qkv: np.ndarray, z: np.ndarray, a: np.ndarray, b: np.ndarray,
                                conv_w: np.ndarray, A_log: np.ndarray, dt_bias: np.ndarray, norm_w: np.ndarray,
                                dtype: str, conv_state: np.ndarray, rec_state: np.ndarray,
                                accepted: np.ndarray):
    """One speculative-decode step with per-row rollback, in the reference's
    terms: the T-token draft runs through the token-by-token mixer with a
    checkpoint after every draft token (speculative.py:778-798 records
    positions prev_seen+1 .. prev_seen+T; local offsets 1..T here), then row b
    continues from the checkpoint of its accepted count a_b
    (select_batch_item(total_valid_tokens=prev_seen + a_b), cache.py:199-244,
    which copies conv_checkpoints / recurrent_checkpoints at that position), or
    from the state before the draft when a_b = 0 (extract_checkpoint at
    past_seen_tokens, cache.py:133-134, which clones the pre-draft cache).
    Returns (gated-norm output [B, T, Hv*dv], conv state, recurrent state)."""
    B, T, _ = mixed_qkv.shape
    out, _, _, conv_cps, rec_cps = mixer_forward(shape, mixed_qkv, z, a, b, conv_w, A_log, dt_bias, norm_w,
                                                 dtype, conv_state, rec_state, chunk=False,
                                                 checkpoint_offsets=list(range(1, T + 1)))
    new_conv = conv_state.copy()
    new_rec = rec_state.copy()
    for row in range(B):
        acc = int(accepted[row])
        if not 0 <= acc <= T:
            raise KeyError(f"checkpoint offset {acc} not recorded")
        if acc > 0:
            new_conv[row] = conv_cps[acc][row]
            new_rec[row] = rec_cps[acc][row]
    return out, new_conv, new_rec
