"""Pipeline parallelism inside one box: contiguous layer stages, boundary activations over
``torch.distributed`` point-to-point (NCCL p2p on GPUs, gloo on CPU), overlapped with
compute across micro-batches.

Decode step of one rank for a batch split into M micro-batches (schedule is a
forward-only GPipe: stage s runs micro-batch m in slot s + m):

    post irecv(m=0)                                   (not first stage)
    for m in 0..M-1:
        wait irecv(m); post irecv(m+1)                 receive overlaps compute of m
        y_m = stage(m, x_m)                            this stage's layers
        isend(y_m) to the next stage on the comm side  send overlaps compute of m+1
    last stage: token ids of every micro-batch go back to stage 0 (one message)

So one step costs (S + M - 1) stage slots instead of S * M.  Every rank issues
the same collective sequence in the same order (including error paths), as
the process-group rules require.

Reference: the serial contiguous-stage ring of si/worker/stage_runtime.py:2137-2275
(one request strictly serial, no micro-batch overlap); the boundary payload
layout is the stage-ring ``[B, S, H]`` activation (si/transport/stage_tensor.py).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist


@dataclass
class PipeGroup:
    rank: int          # stage index
    size: int          # number of stages
    ranks: list[int]   # global ranks of the stages, in order
    group: dist.ProcessGroup | None = None

    @property
    def is_first(self) -> bool:
        return self.rank == 0

    @property
    def is_last(self) -> bool:
        return self.rank == self.size - 1

    def next(self) -> int:
        return self.ranks[self.rank + 1]

    def prev(self) -> int:
        return self.ranks[self.rank - 1]


class PipelineStage:
    """Runs one stage of a micro-batched forward step."""

    def __init__(self, pg: PipeGroup, stage_fn: Callable[[int, torch.Tensor], torch.Tensor],
                 hidden: int, dtype=torch.bfloat16, device="cpu", monitor=None):
        self.pg = pg
        self.fn = stage_fn
        self.hidden = hidden
        self.dtype = dtype
        self.device = torch.device(device)
        # optional ``parallel.rank_health.RankMonitor``: peers that failed, left or went
        # silent are reported before a step's first send / receive, and a transfer broken by
        # a dead peer raises ``RankFailure`` naming it
        self.monitor = monitor

    def step(self, inputs: list[torch.Tensor] | None, mb_sizes: list[int]) -> list[torch.Tensor] | None:
        """``inputs``: per-micro-batch token ids on the first stage (None elsewhere).
        Returns per-micro-batch outputs of the last stage's ``stage_fn`` on stage 0 (the
        tokens travel back), the last stage's own outputs on the last stage, None elsewhere."""
        if self.monitor is None:
            return self._step(inputs, mb_sizes)
        self.monitor.check()
        with self.monitor.guard():
            return self._step(inputs, mb_sizes)

    def _step(self, inputs, mb_sizes):
        pg = self.pg
        M = len(mb_sizes)
        recv_bufs, recv_reqs = [None] * M, [None] * M
        send_reqs = []

        def post_recv(m):
            buf = torch.empty((mb_sizes[m], self.hidden), dtype=self.dtype, device=self.device)
            recv_bufs[m] = buf
            recv_reqs[m] = dist.irecv(buf, src=pg.prev(), group=pg.group)

        outs = []
        if not pg.is_first and M:
            post_recv(0)
        for m in range(M):
            if pg.is_first:
                x = inputs[m]
            else:
                recv_reqs[m].wait()
                if m + 1 < M:
                    post_recv(m + 1)
                x = recv_bufs[m]
            y = self.fn(m, x)
            if pg.is_last:
                outs.append(y)
            else:
                send_reqs.append(dist.isend(y.contiguous(), dst=pg.next(), group=pg.group))
        for r in send_reqs:
            r.wait()
        if pg.size == 1:
            return outs
        # Token / result return: last stage -> first stage, one message per micro-batch.
        if pg.is_last:
            reqs = [dist.isend(o.contiguous(), dst=pg.ranks[0], group=pg.group) for o in outs]
            for r in reqs:
                r.wait()
            return outs
        if pg.is_first:
            res = []
            for m in range(M):
                b = torch.empty_like(self._result_template(mb_sizes[m]))
                dist.recv(b, src=pg.ranks[-1], group=pg.group)
                res.append(b)
            return res
        return None

    result_shape: Callable[[int], tuple] | None = None
    result_dtype = torch.int64

    def _result_template(self, n: int) -> torch.Tensor:
        shape = self.result_shape(n) if self.result_shape else (n,)
        return torch.empty(shape, dtype=self.result_dtype, device=self.device)


def split_batch(n: int, m: int) -> list[int]:
    base, rem = divmod(n, m)
    return [base + (1 if i < rem else 0) for i in range(m) if base + (1 if i < rem else 0) > 0]
