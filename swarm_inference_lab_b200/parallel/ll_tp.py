"""Tensor-parallel row-parallel projections with the low-latency one-shot all-reduce.

``LLTPComm`` gives every rank a symmetric buffer (CUDA IPC, mapped by every peer).  A
row-parallel projection ``h += allreduce(x @ w.T)`` runs as two kernels: the tcgen05
GEMM writes its partial straight into this rank's buffer, and ``ll_allreduce_norm``
(``csrc/kernels/allreduce_ll.cu``) sends every 16-byte piece of it, with the call's
epoch inside each 8-byte word, to every peer, then reads the peers' words from its own
buffer as soon as their epochs match and sums them in rank order (fp32; every rank gets
the same bits) into the residual stream -- also writing the next block's RMSNorm input
when the model asks for it.  There is no system fence and no separate flag, so the
exchange costs one NVLink crossing.  Prefill-sized calls (more tokens than the buffer
holds) use GEMM + NCCL.  ``all_reduce`` / ``all_gather`` / ``reduce_scatter`` forward to
NCCL.

In groups of more than two ranks the same kernel also has a two-shot exchange
(reduce-scatter to the owner of each 1/world slice of the row, then the owner's finished
slice to every peer): (world-1)/world x 2 of a row leaves each rank per token instead of
(world-1) rows, for a second NVLink crossing.  Which one a group uses is measured once at
set-up on a decode-sized call (the timings are summed over the ranks, so every rank picks
the same); ``SIL_LL_MODE=oneshot|twoshot`` overrides it.

Reference semantics: deterministic rank-ordered all-reduce of row-parallel projections,
si/microsharding/dense.py:600-708.
"""
from __future__ import annotations

import os

import torch

from ..ops import gemm
from ..ops._ext import ext
from ..ops.workspace import get_workspace
from .oneshot_tp import MAX_RANKS, open_symmetric


class LLTPComm:
    kernel = "ll_allreduce_norm"

    def __init__(self, base, device: torch.device, *, max_tokens: int = 128, hidden: int = 4096,
                 mode: str | None = None):
        self.base = base
        self.rank = base.rank
        self.size = base.size
        if self.size > MAX_RANKS:
            raise ValueError(f"the one-shot all-reduce supports up to {MAX_RANKS} ranks")
        if hidden % 8 or hidden > 8192:
            raise ValueError("hidden size must be a multiple of 8 and at most 8192")
        self.device = torch.device(device)
        self.max_tokens = max_tokens
        self.hidden = hidden
        self.max_elems = max_tokens * hidden
        self.ll_off = 256
        # ll[2 parities][8 sources][max_elems / 2 words of 8 bytes]
        self.partial_off = self.ll_off + 2 * MAX_RANKS * self.max_elems * 4
        # argmax words [2 parities][8 sources][max_tokens] x 16 bytes
        self.argmax_off = ((self.partial_off + self.max_elems * 2 + 255) // 256) * 256
        nbytes = self.argmax_off + 2 * MAX_RANKS * max_tokens * 16
        self.local, self.peers, self._opened = open_symmetric(base, self.device, nbytes)
        self._views: dict[tuple[int, int], torch.Tensor] = {}
        torch.cuda.synchronize(self.device)
        base.barrier()
        mode = mode or os.environ.get("SIL_LL_MODE", "auto")
        if mode not in ("auto", "oneshot", "twoshot"):
            raise ValueError(f"SIL_LL_MODE must be auto, oneshot or twoshot, not {mode!r}")
        two_ok = self.size > 1 and (hidden // 8) % self.size == 0
        if mode == "twoshot" and not two_ok:
            raise ValueError("the two-shot exchange needs hidden / 8 divisible by the group size")
        self.two_shot = mode == "twoshot"
        self.tuning: dict | None = None
        if mode == "auto" and two_ok and self.size > 2:
            self.two_shot = self._pick_two_shot()

    def _pick_two_shot(self, tokens: int = 32, iters: int = 20) -> bool:
        """Times both exchanges on a ``tokens``-row call (this rank's CUDA events, summed over
        the group so that every rank takes the same decision); True if two-shot is faster.
        An exchange whose calls left an error in the status word (a bounded peer wait ran
        out) counts as infinitely slow on this rank, so the sum steers every rank to the
        other one; the code is cleared and reported as a warning."""
        import warnings
        T = min(tokens, self.max_tokens)
        part = self._partial(T, self.hidden)
        part.zero_()
        h = torch.zeros(T, self.hidden, dtype=torch.bfloat16, device=self.device)
        ws = get_workspace(self.device)
        ms = []
        for two in (False, True):
            for _ in range(3):
                self._exchange(h, None, 0.0, None, ws.status, two)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(iters):
                self._exchange(h, None, 0.0, None, ws.status, two)
            e.record()
            torch.cuda.synchronize(self.device)
            code = ws.code()
            if code:
                warnings.warn(f"LL all-reduce set-up: the {'two' if two else 'one'}-shot exchange "
                              f"reported status {code}; it will not be used", RuntimeWarning)
                ws.clear_status()
                ms.append(float("inf"))
            else:
                ms.append(s.elapsed_time(e) / iters)
        t = torch.tensor(ms, dtype=torch.float32, device=self.device)
        self.base.all_reduce(t)
        tot = t.tolist()
        self.tuning = {"tokens": T, "oneshot_ms_sum": tot[0], "twoshot_ms_sum": tot[1]}
        if tot[0] == float("inf") and tot[1] == float("inf"):
            raise RuntimeError("LL all-reduce set-up: both exchanges failed on some rank")
        return tot[1] < 0.95 * tot[0]

    def _exchange(self, h, norm_w, eps, x_out, status, two_shot=None):
        ext().ll_allreduce_norm(h, self.peers, self.rank, self.ll_off, self.partial_off,
                                self.max_elems, norm_w, float(eps), x_out, status,
                                self.two_shot if two_shot is None else two_shot)

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
        return T * H <= self.max_elems and H == self.hidden and h.is_contiguous()

    def fused_gemm_allreduce_residual(self, x: torch.Tensor, w: torch.Tensor, h: torch.Tensor):
        """h += allreduce(x @ w.T) over the group; returns None (residual already added)."""
        T, H = x.shape[0], w.shape[0]
        if not self._fits(T, H, h):
            out = gemm.linear(x, w)
            self.base.all_reduce(out)
            h.add_(out)
            return None
        part = self._partial(T, H)
        gemm.linear(x, w, out=part)
        self._exchange(h, None, 0.0, None, get_workspace(x.device).status)
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
        part = self._partial(T, H)
        gemm.linear(x, w, out=part)
        self._exchange(h, norm_w, eps, x_out, get_workspace(x.device).status)

    def partial_buffer(self, T: int, H: int) -> torch.Tensor | None:
        """This rank's partial-sum buffer [T, H] (bf16) for a producer that writes its
        row-parallel output there directly (the MoE combine), or None when it does not fit."""
        if T * H > self.max_elems or H != self.hidden:
            return None
        return self._partial(T, H)

    def allreduce_partial_residual(self, h: torch.Tensor, norm_w: torch.Tensor | None = None,
                                   eps: float = 0.0, x_out: torch.Tensor | None = None) -> None:
        """h += sum over ranks of the partial in ``partial_buffer``; with ``norm_w`` also
        x_out = rmsnorm(h) * norm_w."""
        self._exchange(h, norm_w, eps, x_out, get_workspace(h.device).status)

    def argmax_exchange(self, logits: torch.Tensor, idx: torch.Tensor, vocab_start: int) -> torch.Tensor:
        """Global greedy token per row from each rank's local argmax over its vocabulary shard
        (largest logit, lowest global id on ties), exchanged through peer memory."""
        B = logits.shape[0]
        if B > self.max_tokens:
            return None
        out = torch.empty(B, dtype=torch.int64, device=logits.device)
        ext().ll_argmax_exchange(logits, idx, int(vocab_start), self.peers, self.rank,
                                 self.argmax_off, self.max_tokens, out,
                                 get_workspace(logits.device).status)
        return out

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
