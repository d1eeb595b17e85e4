"""Tensor-parallel communicators.

``NcclComm`` wraps a ``torch.distributed`` NCCL process group (one process per
GPU).  It is the unfused baseline: GEMM, then ``all_reduce``.  The fused
path (``parallel/fused_tp.py``) exposes the same interface plus
``fused_gemm_allreduce`` which performs the row-parallel GEMM and the
reduction over NVLink peer memory in one kernel.

``LocalComm`` is the single-rank identity used at TP=1.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class LocalComm:
    rank = 0
    size = 1
    fused_gemm_allreduce = None

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        return x

    def all_gather(self, x: torch.Tensor) -> torch.Tensor:
        return x[None]

    def reduce_scatter(self, x: torch.Tensor) -> torch.Tensor:
        return x

    def barrier(self) -> None:
        pass


class NcclComm:
    """All-reduce / all-gather over an NCCL group (the baseline TP path)."""

    fused_gemm_allreduce = None

    def __init__(self, group: dist.ProcessGroup | None = None, *, deterministic: bool = False):
        self.group = group
        self.rank = dist.get_rank(group)
        self.size = dist.get_world_size(group)
        # Deterministic mode: all-gather the partials and add them in rank order in fp32, the
        # arithmetic of the one-shot NVLink kernels, so both paths give the same bits.
        self.deterministic = deterministic

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        if self.deterministic and self.size > 1:
            g = self.all_gather(x)
            acc = g[0].float()
            for r in range(1, self.size):
                acc += g[r].float()
            x.copy_(acc.to(x.dtype))
            return x
        dist.all_reduce(x, group=self.group)
        return x

    def all_reduce_residual(self, partial: torch.Tensor, h: torch.Tensor) -> None:
        """h += sum over ranks of ``partial``; in deterministic mode the fp32 rank-ordered
        sum is added to h before the single rounding to h's dtype."""
        if self.deterministic and self.size > 1:
            g = self.all_gather(partial)
            acc = g[0].float()
            for r in range(1, self.size):
                acc += g[r].float()
            h.copy_((h.float() + acc).to(h.dtype))
            return
        self.all_reduce(partial)
        h.add_(partial)

    def all_gather(self, x: torch.Tensor) -> torch.Tensor:
        out = torch.empty((self.size,) + tuple(x.shape), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(out, x.contiguous(), group=self.group)
        return out

    def reduce_scatter(self, x: torch.Tensor) -> torch.Tensor:
        """Sum over ranks of ``x`` [size * n, ...]; returns this rank's ``[n, ...]`` slice."""
        out = torch.empty((x.shape[0] // self.size,) + tuple(x.shape[1:]), dtype=x.dtype,
                          device=x.device)
        dist.reduce_scatter_tensor(out, x.contiguous(), group=self.group)
        return out

    def barrier(self) -> None:
        dist.barrier(group=self.group)
