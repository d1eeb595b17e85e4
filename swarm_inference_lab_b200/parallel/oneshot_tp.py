"""Tensor-parallel row-parallel projections with a one-shot NVLink all-reduce.

``OneShotTPComm`` gives every rank a symmetric buffer (CUDA IPC, mapped by every
peer).  A row-parallel projection ``h += allreduce(x @ w.T)`` then runs as two
kernels: the tcgen05 GEMM writes its partial straight into this rank's buffer, and
``oneshot_allreduce`` (``csrc/kernels/allreduce.cu``) has every CTA push its slice of
the partial into every peer's receive slot with 16-byte NVLink stores, raise a per-slice
flag, wait for the peers' flags, and sum the slice in rank order (fp32; all ranks obtain
identical sums) into the residual stream.  Receive slots alternate by epoch parity, so one
flag exchange per call suffices.  Prefill-sized calls (more tokens than the buffer holds) use GEMM +
NCCL.  ``all_reduce`` / ``all_gather`` / ``reduce_scatter`` forward to NCCL.

The model calls ``fused_gemm_allreduce_residual`` (the same hook as the fused
GEMM+all-reduce communicator), so either communicator can be plugged in.

Reference semantics: deterministic rank-ordered all-reduce of row-parallel
projections, si/microsharding/dense.py:600-708.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import gemm
from ..ops._ext import ext
from ..ops.workspace import get_workspace

MAX_RANKS = 8
MAX_CTAS = 256


def open_symmetric(base, device: torch.device, nbytes: int):
    """Allocates a zeroed ``nbytes`` buffer on this rank and maps every peer's buffer
    (CUDA IPC).  Returns ``(local, peers, opened)``: this rank's pointer, every rank's
    pointer in rank order, and the peer mappings to close."""
    e = ext()
    dev = torch.device(device).index
    local = e.symm_alloc(nbytes, dev)
    handles = [None] * base.size
    dist.all_gather_object(handles, (base.rank, e.ipc_handle(local)), group=base.group)
    peers = [0] * base.size
    opened = []
    for r, h in handles:
        if r == base.rank:
            peers[r] = local
        else:
            p = e.ipc_open(h, dev)
            peers[r] = p
            opened.append(p)
    return local, peers, opened


class OneShotTPComm:
    def __init__(self, base, device: torch.device, *, max_tokens: int = 128, hidden: int = 4096):
        self.base = base
        self.rank = base.rank
        self.size = base.size
        if self.size > MAX_RANKS:
            raise ValueError(f"one-shot all-reduce supports up to {MAX_RANKS} ranks")
        self.device = torch.device(device)
        self.max_tokens = max_tokens
        self.hidden = hidden
        self.flags_off = 256
        self.partial_off = ((self.flags_off + MAX_RANKS * MAX_CTAS * 4 + 255) // 256) * 256
        self.max_elems = max_tokens * hidden
        self.recv_off = ((self.partial_off + self.max_elems * 2 + 255) // 256) * 256
        nbytes = self.recv_off + 2 * MAX_RANKS * self.max_elems * 2
        self.local, self.peers, self._opened = open_symmetric(base, self.device, nbytes)
        self._views: dict[tuple[int, int], torch.Tensor] = {}
        torch.cuda.synchronize(self.device)
        base.barrier()

    # NCCL collectives (prefill path and plumbing)
    def all_reduce(self, x):
        return self.base.all_reduce(x)

    def all_gather(self, x):
        return self.base.all_gather(x)

    def reduce_scatter(self, x):
        return self.base.reduce_scatter(x)

    def barrier(self):
        self.base.barrier()

    def _partial(self, T: int, H: int) -> torch.Tensor:
        v = self._views.get((T, H))
        if v is None:
            v = ext().symm_tensor(self.local, self.partial_off, T, H, self.device.index)
            self._views[(T, H)] = v
        return v

    def fused_gemm_allreduce_residual(self, x: torch.Tensor, w: torch.Tensor, h: torch.Tensor):
        """h += allreduce(x @ w.T) over the group; returns None (residual already added)."""
        T, H = x.shape[0], w.shape[0]
        if T * H > self.max_elems or T > self.max_tokens or not h.is_contiguous():
            out = gemm.linear(x, w)
            self.base.all_reduce(out)
            h.add_(out)
            return None
        part = self._partial(T, H)
        gemm.linear(x, w, out=part)
        ext().oneshot_allreduce(h, self.peers, self.rank, self.flags_off, self.recv_off,
                                self.partial_off, self.max_elems, get_workspace(x.device).status)
        return None

    def fused_gemm_allreduce_residual_norm(self, x: torch.Tensor, w: torch.Tensor, h: torch.Tensor,
                                           norm_w: torch.Tensor, eps: float, x_out: torch.Tensor):
        """h += allreduce(x @ w.T); x_out = rmsnorm(h) * norm_w -- the next block's input,
        produced by the all-reduce kernel itself (one CTA per token row)."""
        T, H = x.shape[0], w.shape[0]
        if T * H > self.max_elems or T > self.max_tokens or not h.is_contiguous() or H % 8:
            self.fused_gemm_allreduce_residual(x, w, h)
            from ..ops import norm
            norm.rmsnorm(h, norm_w, eps, out=x_out)
            return
        part = self._partial(T, H)
        gemm.linear(x, w, out=part)
        ext().oneshot_allreduce_norm(h, self.peers, self.rank, self.flags_off, self.recv_off,
                                     self.partial_off, self.max_elems, norm_w, float(eps), x_out,
                                     get_workspace(x.device).status)

    fused_gemm_allreduce = None

    def close(self):
        e = ext()
        torch.cuda.synchronize(self.device)
        self._views.clear()
        for p in self._opened:
            e.ipc_close(p)
        self._opened = []
        if self.local:
            self.base.barrier()
            e.symm_free(self.local)
            self.local = 0
