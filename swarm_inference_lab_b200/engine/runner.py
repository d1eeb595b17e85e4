"""Forward-pass execution for one rank: eager varlen prefill and CUDA-graph decode.

Decode steps are captured once per batch-size bucket into a CUDA graph that
runs every layer, the LM head, greedy selection and a device-side "advance"
(next ids = sampled ids, positions/lengths + 1, next KV slots from the block
table).  A host-driven step overwrites the graph's static inputs from one
pinned staging buffer before replay; a device-driven loop (benchmarks) just
replays, the advance feeding the next step without a host round trip.

Reference: manual CUDA-graph capture/replay per decode position with a
memory admission check (si/model/qwen3_engine.py:154-203, 599-690;
si/execution/qwen3_stage.py:104-188).  Here one graph serves every position
because positions, lengths and slots are device inputs, not constants.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from ..models.dense import ForwardBatch
from ..ops import attention as attn_ops
from .kv_cache import PAGE, PagedKVCache

BUCKETS = (1, 2, 4, 8, 16, 32, 48, 64, 96, 128)


def prefill_host_batch(ids: list[list[int]], starts: list[int], pages: list[list[int]],
                       max_pages: int) -> dict:
    """Host-side arrays of a varlen prefill batch, built with array operations (a 32 x 2048
    token batch is 65536 rows; per-token Python loops cost tens of milliseconds of TTFT):
    flat token ids, absolute positions, KV-cache slots (page * PAGE + offset), per-sequence
    context lengths, the block table and the cumulative query offsets."""
    B = len(ids)
    lens = np.fromiter((len(x) for x in ids), dtype=np.int64, count=B)
    cu = np.zeros(B + 1, dtype=np.int64)
    np.cumsum(lens, out=cu[1:])
    flat = (np.concatenate([np.asarray(x, dtype=np.int64) for x in ids]) if B
            else np.zeros(0, dtype=np.int64))
    st = np.asarray(starts, dtype=np.int64)
    seq_of_row = np.repeat(np.arange(B), lens)
    pos = np.arange(int(cu[-1]), dtype=np.int64) - cu[:-1][seq_of_row] + st[seq_of_row]
    bt = np.zeros((B, max_pages), dtype=np.int64)
    for i, pg in enumerate(pages):
        bt[i, :len(pg)] = pg
    slots = bt[seq_of_row, pos // PAGE] * PAGE + pos % PAGE
    return {"ids": flat, "positions": pos, "slots": slots, "seq_lens": st + lens,
            "block_table": bt, "cu": cu, "max_q_len": int(lens.max()) if B else 0}


def bucket_for(n: int) -> int:
    for b in BUCKETS:
        if n <= b:
            return b
    raise ValueError(f"decode batch {n} exceeds the largest bucket {BUCKETS[-1]}")


@dataclass
class DecodeGraph:
    bsz: int
    graph: torch.cuda.CUDAGraph | None
    ids: torch.Tensor
    meta: torch.Tensor          # int32 [3, bsz]: positions, slots, seq_lens
    valid: torch.Tensor         # bool [bsz]
    block_table: torch.Tensor   # int32 [bsz, max_pages]
    out: torch.Tensor           # int64 [bsz]
    fb: ForwardBatch
    host_ids: torch.Tensor      # pinned staging
    host_meta: torch.Tensor
    host_bt: torch.Tensor
    host_out: torch.Tensor
    n_valid: int = -1


class ModelRunner:
    def __init__(self, model, kv: PagedKVCache, *, max_seq_len: int, use_cuda_graphs: bool = True):
        self.model = model
        self.kv = kv
        self.device = kv.device
        self.max_pages = (max_seq_len + PAGE - 1) // PAGE
        self.use_graphs = use_cuda_graphs
        self.graphs: dict[int, DecodeGraph] = {}
        self.sm_count = torch.cuda.get_device_properties(self.device).multi_processor_count
        self.stream = torch.cuda.current_stream(self.device)

    # ------------------------------------------------------------ prefill
    def prefill(self, ids: list[list[int]], starts: list[int], pages: list[list[int]], *,
                all_rows: bool = False) -> torch.Tensor:
        """Varlen prefill: sequence i appends ``ids[i]`` at positions ``starts[i]..``.
        Returns the greedy token of each sequence's last row (device int64), or of every
        row with ``all_rows`` (multi-token verification for speculative decoding)."""
        dev = self.device
        h = prefill_host_batch(ids, starts, pages, self.max_pages)
        to = lambda a, dt: torch.from_numpy(a).to(dt).to(dev, non_blocking=True)  # noqa: E731
        fb = ForwardBatch(
            ids=to(h["ids"], torch.int64),
            positions=to(h["positions"], torch.int32),
            slots=to(h["slots"], torch.int32),
            seq_lens=to(h["seq_lens"], torch.int32),
            block_table=to(h["block_table"], torch.int32),
            last_idx=(torch.arange(int(h["cu"][-1]), dtype=torch.int64).to(dev, non_blocking=True)
                      if all_rows else to(h["cu"][1:] - 1, torch.int64)),
            is_decode=False,
            cu_q=to(h["cu"], torch.int32),
            max_q_len=int(h["max_q_len"]),
        )
        return self.model.forward(fb, self.kv)

    # ------------------------------------------------------------ decode
    def _make_graph(self, bsz: int) -> DecodeGraph:
        dev = self.device
        ids = torch.zeros(bsz, dtype=torch.int64, device=dev)
        meta = torch.zeros((3, bsz), dtype=torch.int32, device=dev)
        meta[1].fill_(-1)
        meta[2].fill_(1)
        valid = torch.zeros(bsz, dtype=torch.bool, device=dev)
        bt = torch.zeros((bsz, self.max_pages), dtype=torch.int32, device=dev)
        out = torch.zeros(bsz, dtype=torch.int64, device=dev)
        if hasattr(self.model, "decode_splits"):
            splits = self.model.decode_splits(bsz, self.max_pages, self.sm_count)
        else:
            splits = attn_ops.decode_splits(bsz, self.model.num_kv_local, self.max_pages,
                                            self.sm_count)
        fb = ForwardBatch(ids=ids, positions=meta[0], slots=meta[1], seq_lens=meta[2], block_table=bt,
                          last_idx=torch.arange(bsz, dtype=torch.int64, device=dev), is_decode=True,
                          decode_splits=splits)
        pin = dict(pin_memory=True)
        dg = DecodeGraph(bsz, None, ids, meta, valid, bt, out, fb,
                         torch.zeros(bsz, dtype=torch.int64, **pin),
                         torch.zeros((3, bsz), dtype=torch.int32, **pin),
                         torch.zeros((bsz, self.max_pages), dtype=torch.int32, **pin),
                         torch.zeros(bsz, dtype=torch.int64, **pin))
        return dg

    def _step_body(self, dg: DecodeGraph) -> None:
        tok = self.model.forward(dg.fb, self.kv)
        dg.out.copy_(tok)
        # Device-side advance so back-to-back replays need no host round trip.
        dg.ids.copy_(tok)
        pos = dg.meta[0]
        pos.add_(dg.valid.to(torch.int32))
        dg.meta[2].add_(dg.valid.to(torch.int32))
        page_idx = torch.clamp(pos // PAGE, max=self.max_pages - 1).to(torch.int64)
        page = dg.block_table.gather(1, page_idx[:, None]).squeeze(1)
        nxt = page * PAGE + pos % PAGE
        dg.meta[1].copy_(torch.where(dg.valid, nxt, torch.full_like(nxt, -1)))

    def graph_for(self, bsz: int) -> DecodeGraph:
        dg = self.graphs.get(bsz)
        if dg is not None:
            return dg
        dg = self._make_graph(bsz)
        if self.use_graphs:
            # Warm up on a side stream (lazy init, workspace allocation), then capture.
            s = torch.cuda.Stream(self.device)
            s.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(s):
                for _ in range(2):
                    self._step_body(dg)
            torch.cuda.current_stream(self.device).wait_stream(s)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                self._step_body(dg)
            dg.graph = g
            dg.meta.zero_()
            dg.meta[1].fill_(-1)
            dg.meta[2].fill_(1)
        self.graphs[bsz] = dg
        return dg

    def replay(self, dg: DecodeGraph) -> None:
        if dg.graph is not None:
            dg.graph.replay()
        else:
            self._step_body(dg)

    def decode(self, ids: list[int], positions: list[int], pages: list[list[int]]) -> list[int]:
        """Host-driven decode step: stage inputs (pinned H2D), replay, read tokens back."""
        n = len(ids)
        dg = self.graph_for(bucket_for(n))
        self.stage_decode_inputs(dg, ids, positions, pages)
        self.replay(dg)
        dg.host_out.copy_(dg.out, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return dg.host_out[:n].tolist()

    def stage_decode_inputs(self, dg: DecodeGraph, ids, positions, pages) -> int:
        """Fill the pinned staging buffers (numpy views, no per-element torch ops) and
        copy them to the graph inputs.  Returns the host->device bytes copied."""
        n = len(ids)
        hi, hm, hb = dg.host_ids.numpy(), dg.host_meta.numpy(), dg.host_bt.numpy()
        pos = np.asarray(positions, dtype=np.int64)
        hi[:] = 0
        hi[:n] = np.asarray(ids, dtype=np.int64)
        hm[0, :] = 0
        hm[1, :] = -1
        hm[2, :] = 1
        hm[0, :n] = pos
        hm[2, :n] = pos + 1
        for i in range(n):
            row = pages[i]
            hb[i, : len(row)] = row
            hm[1, i] = row[positions[i] // PAGE] * PAGE + positions[i] % PAGE
        dg.ids.copy_(dg.host_ids, non_blocking=True)
        dg.meta.copy_(dg.host_meta, non_blocking=True)
        dg.block_table.copy_(dg.host_bt, non_blocking=True)
        if dg.n_valid != n:
            dg.valid.copy_(torch.arange(dg.bsz) < n)
            dg.n_valid = n
        return dg.host_ids.numel() * 8 + dg.host_meta.numel() * 4 + dg.host_bt.numel() * 4
