"""Fused expert-parallel dispatch / combine over NVLink peer memory.

``FusedEPComm`` gives every rank of an EP group a symmetric buffer (CUDA IPC,
mapped by every peer; layout in ``csrc/include/sil/ep.h`` and
``csrc/kernels/ep.cu``).  A decode MoE layer then moves tokens without NCCL:

1. ``dispatch``: each rank routes its own tokens, quantises them to e4m3 with
   1x128 scales and pushes rows, scales, expert ids and weights into every
   rank's receive slots (P2P stores), then raises its dispatch flag everywhere;
2. ``recv_map`` / ``gather``: each expert owner waits for every source, picks
   the assignments of its local experts and copies their e4m3 rows into expert
   order for the grouped fp8 GEMMs;
3. ``down_scatter``: the grouped down projection multiplies each output row by
   its routing weight and stores it directly into the token owner's combine
   slot (the combine is fused into the GEMM epilogue);
4. ``combine``: each rank waits for every owner and adds its tokens' slots to
   the residual stream in slot order (deterministic).

Prefill-sized calls (more tokens than the buffer holds) use the NCCL path of
the model (all-gather + reduce-scatter); ``all_gather`` / ``reduce_scatter`` /
``all_reduce`` forward to the NCCL communicator.

Reference semantics: expert ownership and the dispatch / return plans of
si/microsharding/moe.py:153-548.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops._ext import ext
from ..ops.workspace import get_workspace

MAX_EP = 8


def _align(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


class FusedEPComm:
    def __init__(self, base, device: torch.device, *, max_tokens: int, hidden: int, top_k: int):
        self.base = base
        self.rank = base.rank
        self.size = base.size
        if self.size > MAX_EP:
            raise ValueError(f"fused EP supports up to {MAX_EP} ranks")
        if hidden % 128:
            raise ValueError("fused EP needs hidden % 128 == 0")
        self.device = torch.device(device)
        self.max_tokens = max_tokens
        self.hidden = hidden
        self.top_k = top_k
        W, Tm, H, k = self.size, max_tokens, hidden, top_k
        off = 256
        dflag = off
        off = _align(off + 2 * 8 * 4)
        cflag = off
        off = _align(off + 2 * 8 * 4)
        rows = off
        off = _align(off + 2 * W * Tm * H)
        scales = off
        off = _align(off + 2 * W * Tm * (H // 128) * 4)
        ids = off
        off = _align(off + 2 * W * Tm * k * 4)
        wts = off
        off = _align(off + 2 * W * Tm * k * 4)
        slots = off
        off = _align(off + 2 * Tm * k * H * 2)
        self.offs = [dflag, cflag, rows, scales, ids, wts, slots]
        self.bytes = off
        e = ext()
        dev = self.device.index
        self.local = e.symm_alloc(self.bytes, dev)
        handles = [None] * self.size
        dist.all_gather_object(handles, (self.rank, e.ipc_handle(self.local)), group=base.group)
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

    # NCCL collectives (prefill path and plumbing)
    def all_reduce(self, x):
        return self.base.all_reduce(x)

    def all_gather(self, x):
        return self.base.all_gather(x)

    def reduce_scatter(self, x):
        return self.base.reduce_scatter(x)

    def barrier(self):
        self.base.barrier()

    @property
    def ep_fused(self):
        return self

    def fits(self, T: int) -> bool:
        return 0 < T <= self.max_tokens

    # fused steps
    def dispatch(self, x: torch.Tensor, ids: torch.Tensor, wts: torch.Tensor, e0: int, el: int) -> None:
        if not self.fits(x.shape[0]) or ids.shape[1] != self.top_k or x.shape[1] != self.hidden:
            raise ValueError("fused EP dispatch: batch exceeds the buffer or shape mismatch")
        st = get_workspace(x.device).status
        ext().ep_dispatch(x, ids, wts, self.peers, self.rank, e0, el, self.offs, st)

    def recv_map(self, T: int, e0: int, el: int) -> torch.Tensor:
        out = torch.empty((self.size * T, self.top_k), dtype=torch.int32, device=self.device)
        ext().ep_recv_map(out, self.peers, self.rank, T, self.top_k, self.hidden, e0, el, self.offs,
                          get_workspace(self.device).status)
        return out

    def gather(self, pos: torch.Tensor, offsets: torch.Tensor, T: int, e0: int, el: int):
        """``pos``: each assignment's sorted position (``moe_ops.permute``).  Returns the e4m3
        rows / scales in expert order and the sorted position -> assignment map."""
        N = pos.shape[0]
        xq = torch.empty((N, self.hidden), dtype=torch.uint8, device=self.device)
        xs = torch.empty((N, self.hidden // 128), dtype=torch.float32, device=self.device)
        inv = torch.empty(N, dtype=torch.int32, device=self.device)
        ext().ep_gather(pos, offsets, xq, xs, inv, self.peers, self.rank, T, self.top_k, self.hidden,
                        e0, el, self.offs, get_workspace(self.device).status)
        return xq, xs, inv

    def down_scatter(self, aq, as_, wq, wscale, offsets, el: int, rows_hint: int, inv, T: int,
                     e0: int) -> None:
        ws = get_workspace(self.device)
        ext().gemm_fp8_grouped_scatter(aq, as_, wq, wscale, offsets, el, int(rows_hint), inv,
                                       self.peers, self.rank, T, self.top_k, e0, self.offs, ws.ws,
                                       ws.counters, ws.status)

    def combine(self, h: torch.Tensor, e0: int, el: int) -> None:
        ext().ep_combine(h, self.peers, self.rank, self.top_k, e0, el, self.offs,
                         get_workspace(self.device).status)

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
