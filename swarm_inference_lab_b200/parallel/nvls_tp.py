"""Tensor-parallel row-parallel projections with a two-shot all-reduce through NVSwitch
multicast (NVLS).

``NvlsTPComm`` allocates one symmetric buffer per rank with torch's symmetric-memory
allocator and rendezvous, which also binds the buffers to one multicast object (the
plumbing only; the collective itself is ``nvls_allreduce`` in ``csrc/kernels/nvls.cu``).
A row-parallel projection ``h += allreduce(x @ w.T)`` runs as two kernels: the tcgen05
GEMM writes its partial straight into this rank's buffer, then ``nvls_allreduce`` has
each rank reduce one column slice of every row in the switch (``multimem.ld_reduce``),
broadcast it into every rank's sum buffer (``multimem.st``), add the row to the residual
stream and, fused, compute the next block's RMSNorm input.

``available(group)`` says whether the box offers multicast; the model falls back to
``OneShotTPComm`` / NCCL otherwise.  Prefill-sized calls (more tokens than the buffer
holds) use GEMM + NCCL.  ``all_reduce`` / ``all_gather`` / ``reduce_scatter`` forward to
NCCL.

Reference semantics: the row-parallel all-reduce of si/microsharding/dense.py:600-708.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import gemm
from ..ops._ext import ext
from ..ops.workspace import get_workspace

MAX_RANKS = 8
MAX_ROWS = 256


def _group_name(group) -> str:
    g = group if group is not None else dist.group.WORLD
    return g.group_name


class NvlsTPComm:
    def __init__(self, base, device: torch.device, *, max_tokens: int = 128, hidden: int = 4096):
        import torch.distributed._symmetric_memory as symm
        self.base = base
        self.rank = base.rank
        self.size = base.size
        if not 2 <= self.size <= MAX_RANKS:
            raise ValueError(f"NVLS all-reduce needs 2..{MAX_RANKS} ranks")
        if max_tokens > MAX_ROWS or hidden % (8 * self.size):
            raise ValueError("NVLS all-reduce: at most 256 rows and hidden a multiple of 8 x ranks")
        self.device = torch.device(device)
        self.max_tokens = max_tokens
        self.hidden = hidden
        self.max_elems = max_tokens * hidden
        self.flags1_off = 256
        self.flags2_off = self.flags1_off + MAX_ROWS * MAX_RANKS * 4
        self.partial_off = ((self.flags2_off + MAX_ROWS * MAX_RANKS * 4 + 255) // 256) * 256
        self.sum_off = ((self.partial_off + self.max_elems * 2 + 255) // 256) * 256
        nbytes = self.sum_off + self.max_elems * 2
        self._buf = symm.empty(nbytes, dtype=torch.uint8, device=self.device)
        self._buf.zero_()
        torch.cuda.synchronize(self.device)
        self._hdl = symm.rendezvous(self._buf, _group_name(base.group))
        if not self._hdl.has_multicast_support() or self._hdl.multicast_ptr == 0:
            self._hdl = None
            self._buf = None
            raise RuntimeError("this box offers no NVLink multicast to the group")
        self.mc = int(self._hdl.multicast_ptr)
        self.peers = [int(p) for p in self._hdl.buffer_ptrs]
        self.local = self.peers[self.rank]
        self._views: dict[tuple[int, int], torch.Tensor] = {}
        base.barrier()

    @staticmethod
    def available(base, device) -> bool:
        """True when the group can use NVLS (tries a rendezvous of a small buffer; every
        rank must call it together)."""
        try:
            import torch.distributed._symmetric_memory as symm
            t = symm.empty(256, dtype=torch.uint8, device=device)
            h = symm.rendezvous(t, _group_name(base.group))
            ok = bool(h.has_multicast_support()) and h.multicast_ptr != 0
            del h, t
        except Exception:  # noqa: BLE001 - no symmetric memory / multicast on this box
            ok = False
        flag = torch.tensor([1 if ok else 0], device=device, dtype=torch.int32)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=base.group)
        return bool(flag.item())

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

    def _fits(self, T: int, H: int, h: torch.Tensor) -> bool:
        return (T * H <= self.max_elems and T <= self.max_tokens and h.is_contiguous()
                and H % (8 * self.size) == 0)

    def _reduce(self, h, norm_w=None, eps=0.0, x_out=None):
        ext().nvls_allreduce(h, self.peers, self.mc, self.rank, self.flags1_off, self.flags2_off,
                             self.partial_off, self.sum_off, self.max_elems, norm_w, float(eps),
                             x_out, get_workspace(h.device).status)

    def fused_gemm_allreduce_residual(self, x: torch.Tensor, w: torch.Tensor, h: torch.Tensor):
        """h += allreduce(x @ w.T) over the group; returns None (residual already added)."""
        T, H = x.shape[0], w.shape[0]
        if not self._fits(T, H, h):
            out = gemm.linear(x, w)
            self.base.all_reduce(out)
            h.add_(out)
            return None
        gemm.linear(x, w, out=self._partial(T, H))
        self._reduce(h)
        return None

    def fused_gemm_allreduce_residual_norm(self, x: torch.Tensor, w: torch.Tensor, h: torch.Tensor,
                                           norm_w: torch.Tensor, eps: float, x_out: torch.Tensor):
        """h += allreduce(x @ w.T); x_out = rmsnorm(h) * norm_w, in the all-reduce kernel."""
        T, H = x.shape[0], w.shape[0]
        if not self._fits(T, H, h):
            self.fused_gemm_allreduce_residual(x, w, h)
            from ..ops import norm
            norm.rmsnorm(h, norm_w, eps, out=x_out)
            return
        gemm.linear(x, w, out=self._partial(T, H))
        self._reduce(h, norm_w, eps, x_out)

    fused_gemm_allreduce = None

    def close(self):
        torch.cuda.synchronize(self.device)
        self._views.clear()
        if self._hdl is not None:
            self.base.barrier()      # every rank is done with the buffer before any releases it
            self._hdl = None
            self._buf = None
