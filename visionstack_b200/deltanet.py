"""Drop-in Gated DeltaNet token mixer on sm_100a kernels.

``Qwen3_5GatedDeltaNet`` has the constructor, parameter names and shapes,
``forward`` signature and cache side effects of the reference layer
(ShadowBoxer/models/qwen35/deltanet.py:410-563).  Between the input
projections and ``out_proj`` (library GEMMs) one fused kernel launch of
``libgdn_b200.so`` does the conv, norms, gates, delta rule and gated RMSNorm.

The functional names of the reference module (deltanet.py:566-574) are kept
with the same signatures; they run the same kernels through the C ABI.
Nothing here computes on the CPU: every entry point requires CUDA tensors
and the compiled library.
"""
from __future__ import annotations

import ctypes
from typing import Dict, List, Optional, Sequence, Tuple, Union

import torch
import torch.nn.functional as F
from torch import nn

from . import _lib
from .cache import Qwen3_5HybridCache, is_owned, mark_owned
from .config import _FP8_DTYPES, Qwen3_5RMSNormGated, Qwen3_5TextConfig, _linear
from .slots import StateSlots

_DTYPES = {torch.float32: _lib.GDN_DTYPE_F32, torch.bfloat16: _lib.GDN_DTYPE_BF16}


def _dtype_code(dt: torch.dtype) -> int:
    if dt not in _DTYPES:
        raise TypeError(f"unsupported activation dtype {dt}; the kernels are built for float32 and bfloat16")
    return _DTYPES[dt]


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _require_cuda(*tensors: Optional[torch.Tensor]) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("the Gated DeltaNet kernels need CUDA tensors (there is no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} and {t.device}")
    if dev is None:
        raise RuntimeError("no tensor given")
    return dev


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


# ---------------------------------------------------------------------------
# Functional boundary (deltanet.py:24-407)
# ---------------------------------------------------------------------------

def _workspace(lib, args, device: torch.device) -> Optional[torch.Tensor]:
    """Scratch of the two-kernel chunked prefill (None when the call needs none)."""
    n = lib.gdn_prefill_workspace_bytes(ctypes.byref(args))
    if n < 0:
        _lib.check("gdn_prefill_workspace_bytes", int(n))
    return torch.empty(int(n), dtype=torch.uint8, device=device) if n > 0 else None


def _extract_conv_state_at_offset(mixed_qkv: torch.Tensor, prev_conv_state: Optional[torch.Tensor],
                                  local_offset: int, state_len: int = 3) -> torch.Tensor:
    """Raw inputs of positions [off - state_len, off) of a [B, C, T] tensor,
    padded from the previous conv state or zeros (deltanet.py:24-38).  Pure
    indexing; the fused kernels write these windows themselves."""
    if local_offset >= state_len:
        return mixed_qkv[:, :, local_offset - state_len:local_offset].contiguous()
    if prev_conv_state is not None:
        return torch.cat([prev_conv_state[:, :, local_offset:], mixed_qkv[:, :, :local_offset]], dim=-1).contiguous()
    return F.pad(mixed_qkv[:, :, :local_offset], (state_len - local_offset, 0)).contiguous()


def _causal_conv1d_fn(hidden_states: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
                      activation: str = "silu", conv_state: Optional[torch.Tensor] = None,
                      return_final_state: bool = False
                      ) -> Union[torch.Tensor, Tuple[torch.Tensor, torch.Tensor]]:
    """Causal depthwise conv1d (+ SiLU) on [B, C, T], signature of
    deltanet.py:41-48; runs ``gdn_causal_conv1d``."""
    if bias is not None:
        raise NotImplementedError("conv bias is not supported (the DeltaNet conv has none)")
    if activation not in ("silu", None, ""):
        raise NotImplementedError(f"activation {activation!r} (only silu)")
    w = weight.squeeze(1) if weight.dim() == 3 else weight
    if w.dtype in _FP8_DTYPES:
        w = w.to(torch.bfloat16 if hidden_states.dtype in _FP8_DTYPES else hidden_states.dtype)
    dt = w.dtype
    dev = _require_cuda(hidden_states, w, conv_state)
    B, C, T = hidden_states.shape
    K = w.shape[-1]
    x = hidden_states.to(dt).contiguous()
    w = w.contiguous()
    cs = None if conv_state is None else conv_state.to(dt).contiguous()
    out = torch.empty((B, C, T), dtype=dt, device=dev)
    st = torch.empty((B, C, K - 1), dtype=hidden_states.dtype if dt == hidden_states.dtype else dt,
                     device=dev) if return_final_state else None
    lib = _lib.load()
    with torch.cuda.device(dev):
        _lib.check("gdn_causal_conv1d", lib.gdn_causal_conv1d(
            B, C, T, K, _dtype_code(dt), _ptr(x), _ptr(w), _ptr(cs), _ptr(out), _ptr(st),
            1 if activation else 0, _stream(dev)))
    res = out.to(hidden_states.dtype)
    if return_final_state:
        return res, st.to(hidden_states.dtype)
    return res


def _solve_unit_lower_triangular(ut_system: torch.Tensor, rhs: torch.Tensor) -> torch.Tensor:
    """(I + tril(ut_system, -1))^-1 @ rhs over the last two dimensions, signature of
    deltanet.py:112-114; runs ``gdn_solve_unit_lower_triangular`` (fp32 forward
    substitution; the batch dimensions broadcast as in the reference's matmul)."""
    dev = _require_cuda(ut_system, rhs)
    n = ut_system.shape[-1]
    if ut_system.shape[-2] != n or rhs.shape[-2] != n:
        raise ValueError(f"shapes {tuple(ut_system.shape)} and {tuple(rhs.shape)} do not form an n x n system")
    m = rhs.shape[-1]
    batch = torch.broadcast_shapes(ut_system.shape[:-2], rhs.shape[:-2])
    u = ut_system.to(torch.float32).expand(*batch, n, n).contiguous()
    r = rhs.to(torch.float32).expand(*batch, n, m).contiguous()
    out = torch.empty((*batch, n, m), dtype=torch.float32, device=dev)
    nb = max(1, int(torch.Size(batch).numel()))
    if out.numel() == 0:
        return out.to(torch.result_type(ut_system, rhs))
    lib = _lib.load()
    with torch.cuda.device(dev):
        _lib.check("gdn_solve_unit_lower_triangular",
                   lib.gdn_solve_unit_lower_triangular(u.data_ptr(), r.data_ptr(), out.data_ptr(), nb, n, m,
                                                       _stream(dev)))
    return out.to(torch.result_type(ut_system, rhs))


def _invert_unit_lower_triangular_block(u_blk: torch.Tensor) -> torch.Tensor:
    """(I + tril(u_blk, -1))^-1 over the last two dimensions, signature of
    deltanet.py:93; ``gdn_solve_unit_lower_triangular`` with the identity as
    right-hand side."""
    dev = _require_cuda(u_blk)
    n = u_blk.shape[-1]
    if u_blk.shape[-2] != n:
        raise ValueError(f"shape {tuple(u_blk.shape)} is not square")
    u = u_blk.to(torch.float32).contiguous()
    out = torch.empty_like(u)
    nb = max(1, int(torch.Size(u.shape[:-2]).numel()))
    if out.numel() == 0:
        return out.to(u_blk.dtype)
    lib = _lib.load()
    with torch.cuda.device(dev):
        _lib.check("gdn_solve_unit_lower_triangular",
                   lib.gdn_solve_unit_lower_triangular(u.data_ptr(), None, out.data_ptr(), nb, n, n, _stream(dev)))
    return out.to(u_blk.dtype)


def _delta_rule(query, key, value, g, beta, initial_state, output_final_state, use_qk_l2norm,
                checkpoint_positions, checkpoint_states_out, past_seen_tokens, chunked: bool):
    dt = query.dtype if query.dtype in _DTYPES else torch.float32
    dev = _require_cuda(query, key, value, g, beta, initial_state)
    B, T, H, dk = key.shape
    dv = value.shape[-1]
    q, k, v, gg, bb = (t.to(dt).contiguous() for t in (query, key, value, g, beta))
    s_in = None if initial_state is None else initial_state.to(device=dev, dtype=torch.float32).contiguous()
    s_out = torch.empty((B, H, dk, dv), dtype=torch.float32, device=dev)
    out = torch.empty((B, T, H, dv), dtype=dt, device=dev)
    offs: List[int] = []
    abs_pos: List[int] = []
    if checkpoint_positions and checkpoint_states_out is not None:
        for cp in sorted({int(c) for c in checkpoint_positions}):
            local = cp - int(past_seen_tokens)
            if 1 <= local <= T:
                offs.append(local)
                abs_pos.append(cp)
    ck_buf = torch.empty((len(offs), B, H, dk, dv), dtype=torch.float32, device=dev) if offs else None
    lib = _lib.load()
    arr = _lib.int_array(offs)
    with torch.cuda.device(dev):
        _lib.check("gdn_delta_rule", lib.gdn_delta_rule(
            B, T, H, dk, dv, _dtype_code(dt), _ptr(q), _ptr(k), _ptr(v), _ptr(gg), _ptr(bb), _ptr(s_in),
            _ptr(s_out), _ptr(out), 1 if use_qk_l2norm else 0, 1 if chunked else 0, len(offs),
            ctypes.cast(arr, ctypes.POINTER(ctypes.c_int32)), _ptr(ck_buf), _stream(dev)))
    if ck_buf is not None:
        for i, cp in enumerate(abs_pos):
            checkpoint_states_out[cp] = ck_buf[i]
    out = out.to(query.dtype)
    if output_final_state:
        return out, s_out
    return out


def _recurrent_gated_delta_rule(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, g: torch.Tensor,
                                beta: torch.Tensor, initial_state: Optional[torch.Tensor] = None,
                                output_final_state: bool = False, use_qk_l2norm: bool = True,
                                checkpoint_positions: Optional[Sequence[int]] = None,
                                checkpoint_states_out: Optional[Dict[int, torch.Tensor]] = None,
                                past_seen_tokens: int = 0):
    """Token-by-token delta rule, signature of deltanet.py:165-177."""
    return _delta_rule(query, key, value, g, beta, initial_state, output_final_state, use_qk_l2norm,
                       checkpoint_positions, checkpoint_states_out, past_seen_tokens, chunked=False)


def _chunk_gated_delta_rule(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, g: torch.Tensor,
                            beta: torch.Tensor, chunk_size: int = 64, initial_state: Optional[torch.Tensor] = None,
                            output_final_state: bool = False, use_qk_l2norm: bool = True,
                            checkpoint_positions: Optional[Sequence[int]] = None,
                            checkpoint_states_out: Optional[Dict[int, torch.Tensor]] = None,
                            past_seen_tokens: int = 0):
    """Chunked delta rule, signature of deltanet.py:236-249.  As in the
    reference, a call with an initial state and T <= 8 runs token by token
    (deltanet.py:251-264).  The kernel always works in chunks of 64 (the
    reference shrinks the chunk to 16 / 32 for short inputs; the result is the
    same up to float rounding), so ``chunk_size`` is accepted and ignored."""
    del chunk_size
    chunked = not (initial_state is not None and key.shape[1] <= 8)
    return _delta_rule(query, key, value, g, beta, initial_state, output_final_state, use_qk_l2norm,
                       checkpoint_positions, checkpoint_states_out, past_seen_tokens, chunked=chunked)


# ---------------------------------------------------------------------------
# The layer (deltanet.py:410-563)
# ---------------------------------------------------------------------------

class Qwen3_5GatedDeltaNet(nn.Module):
    """Gated DeltaNet token mixer; same construction, parameters and
    ``forward`` contract as the reference layer.

    Recurrent states this layer allocated for a cache entry are updated in
    place on later calls (set ``inplace_state = False`` to always allocate a
    new state, as the reference does).  A state placed in the cache by anyone
    else is never written.
    """

    def __init__(self, config: Qwen3_5TextConfig, layer_idx: int):
        super().__init__()
        self.hidden_size = config.hidden_size
        self.num_v_heads = config.linear_num_value_heads
        self.num_k_heads = config.linear_num_key_heads
        self.head_k_dim = config.linear_key_head_dim
        self.head_v_dim = config.linear_value_head_dim
        self.key_dim = self.head_k_dim * self.num_k_heads
        self.value_dim = self.head_v_dim * self.num_v_heads
        self.conv_kernel_size = config.linear_conv_kernel_dim
        self.layer_idx = layer_idx
        self.activation = config.hidden_act
        self.layer_norm_epsilon = config.rms_norm_eps
        self.conv_dim = self.key_dim * 2 + self.value_dim
        self.conv1d = nn.Conv1d(self.conv_dim, self.conv_dim, bias=False, kernel_size=self.conv_kernel_size,
                                groups=self.conv_dim, padding=self.conv_kernel_size - 1)
        self.dt_bias = nn.Parameter(torch.ones(self.num_v_heads))
        self.A_log = nn.Parameter(torch.zeros(self.num_v_heads))
        self.norm = Qwen3_5RMSNormGated(self.head_v_dim, eps=self.layer_norm_epsilon)
        self.out_proj = nn.Linear(self.value_dim, self.hidden_size, bias=False)
        self.in_proj_qkv = nn.Linear(self.hidden_size, self.conv_dim, bias=False)
        self.in_proj_z = nn.Linear(self.hidden_size, self.value_dim, bias=False)
        self.in_proj_b = nn.Linear(self.hidden_size, self.num_v_heads, bias=False)
        self.in_proj_a = nn.Linear(self.hidden_size, self.num_v_heads, bias=False)
        self.inplace_state = True
        self.fuse_in_proj = True
        self._in_proj_fused: Optional[torch.Tensor] = None

    # -- helpers -----------------------------------------------------------
    def _act_dtype(self, x: torch.Tensor) -> torch.dtype:
        w = self.in_proj_qkv.weight
        if w.dtype in _FP8_DTYPES:
            return x.dtype if x.dtype in (torch.bfloat16, torch.float16, torch.float32) else torch.bfloat16
        return w.dtype

    def _param_as(self, p: torch.Tensor, dt: torch.dtype) -> torch.Tensor:
        return p if p.dtype == dt else p.to(dt)

    def _fused_in_proj_weight(self) -> Optional[torch.Tensor]:
        """The four input-projection weights as row ranges of one [conv_dim + Hv*dv + 2 Hv, H]
        tensor, or None where one GEMM cannot serve them (fp8 or mixed dtypes / devices, or a row
        length that would leave the outputs' rows off 16-byte boundaries, which the kernels'
        bulk copies need).  On first use the parameters are re-pointed at their row ranges of the
        fused weight (the state dict keeps its names, shapes and values; loading into it writes
        the fused weight); after anything replaces a parameter's storage (``.to``, assignment)
        the next call fuses again."""
        ws = [self.in_proj_qkv.weight, self.in_proj_z.weight, self.in_proj_b.weight, self.in_proj_a.weight]
        if not self.fuse_in_proj or any(w.dtype in _FP8_DTYPES for w in ws) or \
                len({(w.dtype, w.device) for w in ws}) != 1 or ws[0].device.type != "cuda":
            return None
        n = sum(w.shape[0] for w in ws)
        if (n * ws[0].element_size()) % 16:
            return None
        f = self._in_proj_fused
        if f is not None and f.dtype == ws[0].dtype and f.device == ws[0].device and f.shape[0] == n:
            off, ok = 0, True
            for w in ws:
                ok = ok and w.data_ptr() == f[off].data_ptr() and w.is_contiguous()
                off += w.shape[0]
            if ok:
                return f
        with torch.no_grad():
            f = torch.cat([w.detach() for w in ws], 0).contiguous()
            off = 0
            for w in ws:
                w.data = f[off:off + w.shape[0]]
                off += w.shape[0]
        self._in_proj_fused = f
        return f

    def project(self, hidden_states: torch.Tensor):
        """The four input projections (library GEMMs; the reference's _linear dtype rule):
        mixed_qkv [B,T,conv_dim], z [B,T,Hv*dv], b, a [B,T,Hv].  On a GPU they run as one GEMM
        over the fused weight; the outputs are then column ranges of one [B,T,N] tensor (last
        dimension contiguous, rows 16-byte aligned), which the token mixer reads in place."""
        f = self._fused_in_proj_weight()
        if f is None:
            return (_linear(self.in_proj_qkv, hidden_states), _linear(self.in_proj_z, hidden_states),
                    _linear(self.in_proj_b, hidden_states), _linear(self.in_proj_a, hidden_states))
        x = hidden_states if hidden_states.dtype == f.dtype else hidden_states.to(f.dtype)
        y = F.linear(x, f)
        c0 = self.conv_dim
        c1 = c0 + self.value_dim
        c2 = c1 + self.num_v_heads
        return y[..., :c0], y[..., c0:c1], y[..., c1:c2], y[..., c2:]

    def mixer(self, mixed_qkv: torch.Tensor, z: torch.Tensor, b: torch.Tensor, a: torch.Tensor,
              conv_state: Optional[torch.Tensor] = None, rec_state: Optional[torch.Tensor] = None,
              conv_state_out: Optional[torch.Tensor] = None, rec_state_out: Optional[torch.Tensor] = None,
              out: Optional[torch.Tensor] = None, checkpoint_offsets: Sequence[int] = (),
              state_checkpoints: Optional[torch.Tensor] = None, conv_checkpoints: Optional[torch.Tensor] = None,
              token_by_token: Optional[bool] = None, register_kernel: bool = False,
              cuda_core_prefill: bool = False, fused_prefill: bool = False,
              prep_in_kernel_prefill: bool = False) -> torch.Tensor:
        """One launch of the fused token mixer on projection outputs
        (deltanet.py:489-561): returns the gated-norm output [B, T, Hv*dv].

        ``token_by_token`` picks the decode kernel (T <= 8) or the chunked
        kernel; by default the reference's rule applies (a state and T <= 8).
        The chunked form runs as two kernels (a parallel preparation pass into
        a workspace from torch's caching allocator, then the sequential
        pass).  ``register_kernel`` forces the register-tile decode kernel
        instead of the bulk-copy pipelined one, ``prep_in_kernel_prefill``
        the single kernel whose producer warps prepare each chunk in shared
        memory two chunks ahead of the state pass (workspace only for state
        hand-offs), ``fused_prefill`` the older single kernel that prepares
        each chunk on the state's critical path (no workspace),
        ``cuda_core_prefill`` the CUDA-core chunked kernel (same results up to
        float rounding; used by the tests).
        """
        if token_by_token is None:
            token_by_token = rec_state is not None and mixed_qkv.shape[1] <= _lib.GDN_MAX_DECODE_TOKENS
        flags = (_lib.GDN_FLAG_REGISTER_KERNEL if register_kernel else 0) | \
            (_lib.GDN_FLAG_CUDA_CORE_PREFILL if cuda_core_prefill else 0) | \
            (_lib.GDN_FLAG_PREP_IN_KERNEL_PREFILL if prep_in_kernel_prefill else 0)
        args, out, keep = self._mixer_args(mixed_qkv, z, b, a, conv_state, rec_state, conv_state_out,
                                           rec_state_out, out, flags)
        offs = list(checkpoint_offsets)
        arr = _lib.int_array(offs)
        args.num_checkpoints = len(offs)
        args.checkpoint_offsets = ctypes.cast(arr, ctypes.POINTER(ctypes.c_int32))
        args.state_checkpoints = _ptr(state_checkpoints)
        args.conv_checkpoints = _ptr(conv_checkpoints)
        lib = _lib.load()
        with torch.cuda.device(out.device):
            if token_by_token:
                _lib.check("gdn_mixer_decode", lib.gdn_mixer_decode(ctypes.byref(args), _stream(out.device)))
            elif fused_prefill:
                _lib.check("gdn_mixer_prefill", lib.gdn_mixer_prefill(ctypes.byref(args), _stream(out.device)))
            else:
                ws = _workspace(lib, args, out.device)
                _lib.check("gdn_mixer_prefill_ws",
                           lib.gdn_mixer_prefill_ws(ctypes.byref(args), None if ws is None else ws.data_ptr(),
                                                    0 if ws is None else ws.numel(), _stream(out.device)))
        return out

    def mixer_verify(self, mixed_qkv: torch.Tensor, z: torch.Tensor, b: torch.Tensor, a: torch.Tensor,
                     slots: "StateSlots", out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Token mixer of a speculative-decode verify step on per-row state
        slots (``StateSlots``): each row starts from its current slot and the
        states after every draft token land in its free slots; nothing is
        written over the starting state.  Returns the gated-norm output
        [B, T, Hv*dv]; follow with ``slots.accept(counts)``."""
        B, T, _ = mixed_qkv.shape
        if B != slots.batch or T > slots.num_slots - 1:
            raise ValueError(f"draft of {T} tokens for {B} rows does not fit slots of {slots.batch} rows x "
                             f"{slots.num_slots - 1} tokens")
        if slots.conv.dtype != mixed_qkv.dtype:
            raise TypeError(f"conv slots hold {slots.conv.dtype}, activations are {mixed_qkv.dtype}")
        args, out, keep = self._mixer_args(mixed_qkv, z, b, a, slots.conv, slots.state, None, None, out, 0)
        lib = _lib.load()
        with torch.cuda.device(out.device):
            _lib.check("gdn_mixer_verify_slots",
                       lib.gdn_mixer_verify_slots(ctypes.byref(args), slots.table.data_ptr(), slots.num_slots,
                                                  _stream(out.device)))
        slots.last_len = T
        return out

    def verify(self, hidden_states: torch.Tensor, slots: "StateSlots") -> torch.Tensor:
        """Layer output of a speculative-decode verify step: the four
        projections, ``mixer_verify`` and ``out_proj``.  The reference runs the
        same forward on a cache cloned per candidate with a checkpoint after
        every draft token (speculative.py:778-798)."""
        mixed_qkv, z, b, a = self.project(hidden_states)
        return _linear(self.out_proj, self.mixer_verify(mixed_qkv, z, b, a, slots))

    def _mixer_args(self, mixed_qkv, z, b, a, conv_state, rec_state, conv_state_out, rec_state_out, out, flags):
        """Fill a ``gdn_mixer_args`` for one call; returns (args, out, tensors
        that must stay alive until the launch)."""
        B, T, _ = mixed_qkv.shape
        dt = mixed_qkv.dtype
        dev = _require_cuda(mixed_qkv, z, b, a, conv_state, rec_state)
        if mixed_qkv.stride(-1) != 1 or z.stride(-1) != 1 or a.stride(-1) != 1 or b.stride(-1) != 1:
            raise RuntimeError("projection outputs must have a contiguous last dimension")
        if a.stride() != b.stride():
            a, b = a.contiguous(), b.contiguous()
        if z.dim() == 4:
            z = z.reshape(B, T, -1)
        conv_w = self.conv1d.weight
        if conv_w.dtype in _FP8_DTYPES:
            conv_w = conv_w.to(dt)
        conv_w = conv_w.reshape(self.conv_dim, self.conv_kernel_size)
        if conv_w.dtype != dt or self.norm.weight.dtype != dt:
            raise TypeError(f"conv/norm weights must be in the activation dtype {dt}")
        conv_w = conv_w.contiguous()
        A_log = self.A_log.detach().float().contiguous()
        dt_bias = self.dt_bias.detach().float().contiguous()
        normw = self.norm.weight.detach().contiguous()
        if out is None:
            out = torch.empty((B, T, self.value_dim), dtype=dt, device=dev)
        args = _lib.MixerArgs()
        args.batch, args.seq_len = B, T
        args.num_k_heads, args.num_v_heads = self.num_k_heads, self.num_v_heads
        args.head_k_dim, args.head_v_dim = self.head_k_dim, self.head_v_dim
        args.conv_kernel = self.conv_kernel_size
        args.act_dtype = _dtype_code(dt)
        args.norm_eps = float(self.layer_norm_epsilon)
        args.flags = flags
        args.mixed_qkv, args.mixed_stride_b, args.mixed_stride_t = mixed_qkv.data_ptr(), mixed_qkv.stride(0), \
            mixed_qkv.stride(1)
        args.z, args.z_stride_b, args.z_stride_t = z.data_ptr(), z.stride(0), z.stride(1)
        args.a, args.b = a.data_ptr(), b.data_ptr()
        args.ab_stride_b, args.ab_stride_t = a.stride(0), a.stride(1)
        args.conv_weight, args.A_log, args.dt_bias, args.norm_weight = (
            conv_w.data_ptr(), A_log.data_ptr(), dt_bias.data_ptr(), normw.data_ptr())
        if conv_state is not None:
            conv_state = conv_state.to(dt).contiguous()
        args.conv_state_in = _ptr(conv_state)
        args.conv_state_out = _ptr(conv_state_out)
        if rec_state is not None and (rec_state.dtype != torch.float32 or not rec_state.is_contiguous()):
            rec_state = rec_state.float().contiguous()
        args.state_in = _ptr(rec_state)
        args.state_out = _ptr(rec_state_out)
        args.out = out.data_ptr()
        return args, out, (a, b, z, conv_w, A_log, dt_bias, normw, conv_state, rec_state)

    def mixer_plan(self, batch: int, seq_len: int, dtype: torch.dtype, device,
                   token_by_token: bool = True) -> "MixerPlan":
        """Pre-bind this layer's weights and shapes for repeated ``mixer``
        calls (a serving decode loop): each call then only sets pointers."""
        device = torch.device(device)
        if device.type == "cuda" and device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        return MixerPlan(self, batch, seq_len, dtype, device, token_by_token)

    # -- forward -----------------------------------------------------------
    def forward(self, hidden_states: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                cache: Optional[Qwen3_5HybridCache] = None) -> torch.Tensor:
        if attention_mask is not None and attention_mask.ndim == 2:
            hidden_states = hidden_states * attention_mask[:, :, None].to(hidden_states.dtype)
        B, T, _ = hidden_states.shape
        mixed_qkv, z, b, a = self.project(hidden_states)
        dt = mixed_qkv.dtype
        dev = mixed_qkv.device
        L = self.conv_kernel_size - 1
        l = self.layer_idx

        prev_conv = cache.conv_states.get(l) if cache is not None else None
        prev_rec = cache.recurrent_states.get(l) if cache is not None else None
        past = cache.past_seen_tokens if cache is not None else 0
        cps = cache.checkpoint_offsets if (cache is not None and cache.record_checkpoints) else None

        conv_out = rec_out = None
        offs: List[int] = []
        abs_pos: List[int] = []
        st_ck = cv_ck = None
        if cache is not None:
            conv_out = torch.empty((B, self.conv_dim, L), dtype=dt, device=dev)
            if prev_rec is not None and self.inplace_state and is_owned(prev_rec, cache, l) and \
                    prev_rec.dtype == torch.float32 and prev_rec.is_contiguous() and prev_rec.device == dev:
                rec_out = prev_rec
            else:
                rec_out = torch.empty((B, self.num_v_heads, self.head_k_dim, self.head_v_dim),
                                      dtype=torch.float32, device=dev)
            if cps:
                for cp in sorted({int(c) for c in cps}):
                    local = cp - past
                    if 1 <= local <= T:
                        offs.append(local)
                        abs_pos.append(cp)
                if offs:
                    st_ck = torch.empty((len(offs), B, self.num_v_heads, self.head_k_dim, self.head_v_dim),
                                        dtype=torch.float32, device=dev)
                    cv_ck = torch.empty((len(offs), B, self.conv_dim, L), dtype=dt, device=dev)

        core = self.mixer(mixed_qkv, z, b, a, conv_state=prev_conv, rec_state=prev_rec, conv_state_out=conv_out,
                          rec_state_out=rec_out, checkpoint_offsets=offs, state_checkpoints=st_ck,
                          conv_checkpoints=cv_ck)

        if cache is not None:
            cache.conv_states[l] = conv_out
            cache.recurrent_states[l] = mark_owned(rec_out, cache, l)
            for i, cp in enumerate(abs_pos):
                cache.conv_checkpoints.setdefault(cp, {})[l] = cv_ck[i]
                cache.recurrent_checkpoints.setdefault(cp, {})[l] = st_ck[i]
        return _linear(self.out_proj, core)


class MixerPlan:
    """Repeated token-mixer calls with pre-bound weights and shapes.

    Built by ``Qwen3_5GatedDeltaNet.mixer_plan``.  ``__call__`` takes the
    per-step device tensors (projection outputs, states, output) and launches
    the same kernel as ``Qwen3_5GatedDeltaNet.mixer`` with no per-call tensor
    conversions; the C ABI still validates every call.  The layer's
    parameters must not be replaced while the plan is in use.
    """

    def __init__(self, layer: Qwen3_5GatedDeltaNet, batch: int, seq_len: int, dtype: torch.dtype,
                 device: torch.device, token_by_token: bool):
        conv_w = layer.conv1d.weight
        if conv_w.dtype in _FP8_DTYPES:
            conv_w = conv_w.to(dtype)
        self._conv_w = conv_w.detach().reshape(layer.conv_dim, layer.conv_kernel_size).contiguous()
        self._A_log = layer.A_log.detach().float().contiguous()
        self._dt_bias = layer.dt_bias.detach().float().contiguous()
        self._normw = layer.norm.weight.detach().contiguous()
        for t in (self._conv_w, self._A_log, self._dt_bias, self._normw):
            if t.device != device:
                raise RuntimeError("layer parameters must live on the plan's device")
        if self._conv_w.dtype != dtype or self._normw.dtype != dtype:
            raise TypeError(f"conv/norm weights must be in the activation dtype {dtype}")
        a = _lib.MixerArgs()
        a.batch, a.seq_len = batch, seq_len
        a.num_k_heads, a.num_v_heads = layer.num_k_heads, layer.num_v_heads
        a.head_k_dim, a.head_v_dim = layer.head_k_dim, layer.head_v_dim
        a.conv_kernel = layer.conv_kernel_size
        a.act_dtype = _dtype_code(dtype)
        a.norm_eps = float(layer.layer_norm_epsilon)
        a.conv_weight, a.A_log = self._conv_w.data_ptr(), self._A_log.data_ptr()
        a.dt_bias, a.norm_weight = self._dt_bias.data_ptr(), self._normw.data_ptr()
        self._args = a
        self._ref = ctypes.byref(a)
        self._lib = _lib.load()
        self._token_by_token = token_by_token
        self._ws: Optional[torch.Tensor] = None
        self.device = device

    def __call__(self, mixed_qkv: torch.Tensor, z: torch.Tensor, b: torch.Tensor, a: torch.Tensor,
                 conv_state: Optional[torch.Tensor], rec_state: Optional[torch.Tensor],
                 conv_state_out: Optional[torch.Tensor], rec_state_out: Optional[torch.Tensor],
                 out: torch.Tensor, stream: Optional[int] = None) -> torch.Tensor:
        g = self._args
        g.mixed_qkv, g.mixed_stride_b, g.mixed_stride_t = mixed_qkv.data_ptr(), mixed_qkv.stride(0), \
            mixed_qkv.stride(1)
        g.z, g.z_stride_b, g.z_stride_t = z.data_ptr(), z.stride(0), z.stride(1)
        g.a, g.b, g.ab_stride_b, g.ab_stride_t = a.data_ptr(), b.data_ptr(), a.stride(0), a.stride(1)
        g.conv_state_in = None if conv_state is None else conv_state.data_ptr()
        g.conv_state_out = None if conv_state_out is None else conv_state_out.data_ptr()
        g.state_in = None if rec_state is None else rec_state.data_ptr()
        g.state_out = None if rec_state_out is None else rec_state_out.data_ptr()
        g.out = out.data_ptr()
        sh = torch.cuda.current_stream(self.device).cuda_stream if stream is None else stream
        if self._token_by_token:
            st = self._lib.gdn_mixer_decode(self._ref, sh)
            if st:
                _lib.check("gdn_mixer_decode", st)
            return out
        if self._ws is None:
            self._ws = _workspace(self._lib, g, self.device)
            if self._ws is None:
                self._ws = torch.empty(0, dtype=torch.uint8, device=self.device)
        st = self._lib.gdn_mixer_prefill_ws(self._ref, self._ws.data_ptr() if self._ws.numel() else None,
                                            self._ws.numel(), sh)
        if st:
            _lib.check("gdn_mixer_prefill_ws", st)
        return out


__all__ = [
    "MixerPlan",
    "_extract_conv_state_at_offset",
    "_causal_conv1d_fn",
    "_recurrent_gated_delta_rule",
    "_chunk_gated_delta_rule",
    "_solve_unit_lower_triangular",
    "_invert_unit_lower_triangular_block",
    "Qwen3_5GatedDeltaNet",
]
