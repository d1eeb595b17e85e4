"""Fused tensor-parallel communication over NVLink peer memory.

``FusedTPComm`` gives every rank of a TP group a symmetric buffer (same
size and layout on every GPU, exported with CUDA IPC and mapped by every
peer).  Row-parallel projections then run as ONE kernel per rank
(``csrc/kernels/gemm_bf16_impl.cuh``, epilogue ``kEpiAllReduce``): the
tcgen05 GEMM computes the rank's partial tile, stores it into slot
``[epoch parity][rank]`` of every peer's buffer with P2P stores, raises the
tile's flag on every peer, and finally each CTA reduces the tiles it owns
in rank order (fp32 sum of bf16 partials, like the reference's
deterministic rank-ordered reduction) and adds the residual in place.
Waits on peer flags are bounded by a deadline and report through the
device status word.

Decode-sized calls (<= 128 tokens) take the fused path; larger calls
(prefill) fall back to GEMM + NCCL all-reduce.  ``all_reduce`` /
``all_gather`` always use NCCL (the baseline path, and PP/argmax plumbing).

Reference semantics: row-parallel o/down projections with a deterministic
rank-ordered all-reduce, si/microsharding/dense.py:600-708, 734-742.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops._ext import ext
from ..ops import gemm
from ..ops.workspace import get_workspace

MAX_TP = 8
STATE_BYTES = 256


class FusedTPComm:
    def __init__(self, base, device: torch.device, *, max_tokens: int = 128, hidden: int = 4096):
        self.base = base
        self.rank = base.rank
        self.size = base.size
        if self.size > MAX_TP:
            raise ValueError(f"fused TP supports up to {MAX_TP} ranks")
        self.device = torch.device(device)
        self.max_tokens = min(max_tokens, 128)
        self.max_hidden = hidden
        self.max_tiles = (hidden + 127) // 128
        self.flags_off = STATE_BYTES
        flags_bytes = 2 * MAX_TP * self.max_tiles * 4
        self.slots_off = ((self.flags_off + flags_bytes + 255) // 256) * 256
        slots_bytes = 2 * MAX_TP * self.max_tokens * self.max_hidden * 2
        self.bytes = self.slots_off + slots_bytes
        e = ext()
        dev = self.device.index
        self.local = e.symm_alloc(self.bytes, dev)
        handle = e.ipc_handle(self.local)
        handles = [None] * self.size
        dist.all_gather_object(handles, (self.rank, handle), group=base.group)
        self.peers = [0] * self.size
        self._opened = []
        for r, h in handles:
            if r == self.rank:
                self.peers[r] = self.local
            else:
                p = e.ipc_open(h, dev)
                self.peers[r] = p
                self._opened.append(p)
        torch.cuda.synchronize(self.device)
        base.barrier()

    # NCCL-backed collectives (baseline path and small plumbing).
    def all_reduce(self, x):
        return self.base.all_reduce(x)

    def all_gather(self, x):
        return self.base.all_gather(x)

    def reduce_scatter(self, x):
        return self.base.reduce_scatter(x)

    def barrier(self):
        self.base.barrier()

    def fused_gemm_allreduce_residual(self, x: torch.Tensor, w: torch.Tensor, h: torch.Tensor):
        """h += allreduce(x @ w.T) over the group; returns None (residual already added)."""
        if x.shape[0] > self.max_tokens or w.shape[0] > self.max_hidden:
            out = gemm.linear(x, w)
            self.base.all_reduce(out)
            h.add_(out)
            return None
        ws = get_workspace(x.device)
        ext().gemm_allreduce(x, w, h, self.peers, self.rank, self.max_tiles, self.max_tokens,
                             self.max_hidden, self.flags_off, self.slots_off, ws.ws, ws.counters,
                             ws.status)
        return None

    fused_gemm_allreduce = None  # the residual-fused variant above is the one the model uses

    def close(self):
        e = ext()
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            e.ipc_close(p)
        self._opened = []
        if self.local:
            self.base.barrier()
            e.symm_free(self.local)
            self.local = 0
