"""One-shot all-reduce of small bf16 tensors over NVLink peer memory (``gdn_peer_allreduce_bf16``).

The exchange step of the value-head-sharded layers sums row-parallel partial outputs of a few
hundred KB per decode step (``out_proj`` after the token mixer; ``o_proj`` and ``down_proj`` in
the sharded stack).  A ring all-reduce of that size is bound by its per-step latency; here every
rank stages its partial in memory that every other rank has mapped (CUDA IPC: plain peer loads
and stores over NVLink, no multicast), one flag exchange per call tells the ranks that all
partials are there, and each rank sums all of them itself: one launch, one NVLink round trip.
The reference runs on one GPU and has no counterpart.

Every rank of the group must create the object and then call it the same number of times in the
same order (calls can be captured in CUDA graphs).  Tensors larger than the staging capacity are
summed by the process group's own all-reduce (NCCL) instead.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib


class PeerAllReduce:
    """Sum of a bf16 tensor across the ranks of ``group`` (one GPU per rank, one node).

    ``max_elems``: staging capacity per call (elements); ``nblocks``: thread blocks per call, each
    with its own flags, the same on every rank.
    """

    def __init__(self, group=None, max_elems: int = 1 << 20, nblocks: int = 32,
                 device: Optional[torch.device] = None):
        import torch.distributed as dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > _lib.GDN_PEER_MAX_RANKS:
            raise ValueError(f"at most {_lib.GDN_PEER_MAX_RANKS} ranks")
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.cap = int(max_elems) // 8 * 8
        self.nblocks = int(nblocks)
        self._own: Optional[int] = None
        self._opened = []
        lib = _lib.load()
        with torch.cuda.device(self.device):
            nbytes = int(lib.gdn_peer_staging_bytes(self.world, self.nblocks, self.cap))
            if nbytes < 0:
                _lib.check("gdn_peer_staging_bytes", nbytes)
            own = ctypes.c_void_p()
            _lib.check("gdn_peer_staging_alloc", lib.gdn_peer_staging_alloc(nbytes, ctypes.byref(own)))
            self._own = own.value
            handle = (ctypes.c_char * _lib.GDN_IPC_HANDLE_BYTES)()
            _lib.check("gdn_ipc_get_handle", lib.gdn_ipc_get_handle(self._own, handle))
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
            g = _lib.PeerGroup()
            g.rank, g.world, g.nblocks, g.cap = self.rank, self.world, self.nblocks, self.cap
            for r in range(self.world):
                if r == self.rank:
                    g.staging[r] = self._own
                    continue
                buf = ctypes.create_string_buffer(handles[r], _lib.GDN_IPC_HANDLE_BYTES)
                ptr = ctypes.c_void_p()
                _lib.check("gdn_ipc_open_handle", lib.gdn_ipc_open_handle(buf, ctypes.byref(ptr)))
                self._opened.append(ptr.value)
                g.staging[r] = ptr.value
            self._group = g
        dist.barrier(group)

    def fits(self, x: torch.Tensor) -> bool:
        """True when ``x`` goes through the peer path: bf16 on this rank's device, a multiple of 8
        elements up to the capacity.  Every input of the decision is the same on every rank of a
        sharded layer (dtype, size), so the ranks never split between this path and another."""
        n = x.numel()
        return x.dtype == torch.bfloat16 and x.device == self.device and n % 8 == 0 and 0 < n <= self.cap

    def __call__(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Sum ``x`` over the ranks into ``out`` (default: in place) on the current stream."""
        if out is None:
            out = x
        if self.world == 1:
            if out.data_ptr() != x.data_ptr():
                out.copy_(x)
            return out
        if not self.fits(x) or out.shape != x.shape or not self.fits(out):
            raise ValueError(f"PeerAllReduce takes bf16 tensors of a multiple of 8 elements up to {self.cap} "
                             f"on {self.device}")

        def direct(t: torch.Tensor) -> bool:
            return t.is_contiguous() and t.data_ptr() % 16 == 0
        src = x if direct(x) else x.contiguous().clone()  # a fresh allocation is 16-byte aligned
        dst = out if direct(out) else torch.empty(out.shape, dtype=out.dtype, device=out.device)
        lib = _lib.load()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check("gdn_peer_allreduce_bf16", lib.gdn_peer_allreduce_bf16(
            ctypes.byref(self._group), src.data_ptr(), dst.data_ptr(), src.numel(), stream))
        if dst is not out:
            out.copy_(dst)
        return out

    def close(self) -> None:
        """Unmap the peers' staging memory and free this rank's (collective: every rank calls it)."""
        import torch.distributed as dist
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)
        lib = _lib.load()
        with torch.cuda.device(self.device):
            for p in self._opened:
                _lib.check("gdn_ipc_close_handle", lib.gdn_ipc_close_handle(p))
            self._opened = []
            dist.barrier(self.group)
            _lib.check("gdn_peer_staging_free", lib.gdn_peer_staging_free(self._own))
        self._own = None


def sum_partials(x: torch.Tensor, peer: Optional[PeerAllReduce], group=None) -> torch.Tensor:
    """Sum ``x`` over the ranks in place: the peer path when it fits, else the group's all-reduce."""
    import torch.distributed as dist
    if peer is not None and peer.fits(x):
        return peer(x)
    dist.all_reduce(x, op=dist.ReduceOp.SUM, group=group)
    return x


__all__ = ["PeerAllReduce", "sum_partials"]
