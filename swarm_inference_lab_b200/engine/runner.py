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
class SamplingState:
    """Per-row sampling inputs of a captured decode graph (device) and their pinned
    staging buffers: temperature, top-k, top-p, repetition penalty, Philox seed and offset
    (the token index), and the token history the repetition penalty looks at."""
    temp: torch.Tensor
    top_k: torch.Tensor
    top_p: torch.Tensor
    penalty: torch.Tensor
    seeds: torch.Tensor
    offsets: torch.Tensor
    history: torch.Tensor       # int64 [bsz, hmax]
    hist_len: torch.Tensor      # int32 [bsz]
    host_f: torch.Tensor        # pinned fp32 [3, bsz]: temp, top_p, penalty
    host_i: torch.Tensor        # pinned int64 [2, bsz]: seeds, offsets
    host_k: torch.Tensor        # pinned int32 [2, bsz]: top_k, hist_len
    host_hist: torch.Tensor     # pinned int64 [bsz, hmax]
    key: tuple | None = None    # requests whose history is on the device


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
    sampling: SamplingState | None = None


class ModelRunner:
    def __init__(self, model, kv: PagedKVCache, *, max_seq_len: int, use_cuda_graphs: bool = True):
        self.model = model
        self.kv = kv
        self.device = kv.device
        self.max_pages = (max_seq_len + PAGE - 1) // PAGE
        self.use_graphs = use_cuda_graphs
        self.graphs: dict[tuple[int, bool], DecodeGraph] = {}
        self.sm_count = torch.cuda.get_device_properties(self.device).multi_processor_count
        self.stream = torch.cuda.current_stream(self.device)
        self.max_seq_len = max_seq_len

    # ------------------------------------------------------------ logits / sampling
    def _full_logits(self, h: torch.Tensor, fb: ForwardBatch) -> torch.Tensor:
        """fp32 logits over the whole vocabulary (gathered over a vocabulary-parallel group)."""
        lg = self.model.logits(h, fb)
        tp = getattr(self.model, "tp", None)
        if tp is not None and tp.size > 1 and getattr(self.model, "w", None) is not None \
                and hasattr(self.model.w, "vocab_start"):
            parts = self.model.comm.all_gather(lg)          # [tp, B, V / tp]
            lg = parts.permute(1, 0, 2).reshape(lg.shape[0], -1).contiguous()
        return lg

    @staticmethod
    def _row_params(sampling: list) -> tuple[list, list, list, list, list]:
        t, k, p, r, sd = [], [], [], [], []
        for sp in sampling:
            if sp is None:
                t.append(0.0), k.append(0), p.append(1.0), r.append(1.0), sd.append(0)
            else:
                t.append(float(sp.temperature)), k.append(int(sp.top_k)), p.append(float(sp.top_p))
                r.append(float(sp.repetition_penalty)), sd.append(int(sp.seed or 0))
        return t, k, p, r, sd

    # ------------------------------------------------------------ prefill
    def prefill(self, ids: list[list[int]], starts: list[int], pages: list[list[int]], *,
                all_rows: bool = False, sampling: list | None = None,
                history: list[list[int]] | None = None) -> torch.Tensor:
        """Varlen prefill: sequence i appends ``ids[i]`` at positions ``starts[i]..``.
        Returns the greedy token of each sequence's last row (device int64), or of every
        row with ``all_rows`` (multi-token verification for speculative decoding).  With
        ``sampling`` (one SamplingParams or None per sequence) the first output token of
        each sequence is drawn instead (token index 0 of its Philox stream); ``history``
        holds the tokens the repetition penalty sees (the prompt)."""
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
        if sampling is None or all_rows:
            return self.model.forward(fb, self.kv)
        from ..ops import sampling as samp_ops
        hid = self.model.forward_hidden(fb, self.kv)
        logits = self._full_logits(hid, fb)
        B = len(ids)
        t, k, p, r, sd = self._row_params(sampling)
        hist = history or [[] for _ in range(B)]
        hmax = max(1, max(len(x) for x in hist))
        hh = np.zeros((B, hmax), dtype=np.int64)
        for i, x in enumerate(hist):
            hh[i, :len(x)] = x
        hl = torch.tensor([len(x) for x in hist], dtype=torch.int32).to(dev)
        return samp_ops.sample(logits, temperature=torch.tensor(t), top_k=torch.tensor(k),
                               top_p=torch.tensor(p), repetition_penalty=torch.tensor(r),
                               history=torch.from_numpy(hh).to(dev), history_len=hl,
                               seeds=torch.tensor(sd, dtype=torch.int64),
                               offsets=torch.zeros(B, dtype=torch.int64))

    # ------------------------------------------------------------ decode
    def _make_graph(self, bsz: int, sampled: bool = False) -> DecodeGraph:
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
        if sampled:
            hmax = self.max_seq_len
            dg.sampling = SamplingState(
                temp=torch.zeros(bsz, dtype=torch.float32, device=dev),
                top_k=torch.zeros(bsz, dtype=torch.int32, device=dev),
                top_p=torch.ones(bsz, dtype=torch.float32, device=dev),
                penalty=torch.ones(bsz, dtype=torch.float32, device=dev),
                seeds=torch.zeros(bsz, dtype=torch.int64, device=dev),
                offsets=torch.zeros(bsz, dtype=torch.int64, device=dev),
                history=torch.zeros((bsz, hmax), dtype=torch.int64, device=dev),
                hist_len=torch.zeros(bsz, dtype=torch.int32, device=dev),
                host_f=torch.zeros((3, bsz), dtype=torch.float32, **pin),
                host_i=torch.zeros((2, bsz), dtype=torch.int64, **pin),
                host_k=torch.zeros((2, bsz), dtype=torch.int32, **pin),
                host_hist=torch.zeros((bsz, hmax), dtype=torch.int64, **pin))
        return dg

    def _step_body(self, dg: DecodeGraph) -> None:
        from ..ops._ext import ext
        st = dg.sampling
        if st is None:
            tok = self.model.forward(dg.fb, self.kv)
        else:
            from ..ops import sampling as samp_ops
            h = self.model.forward_hidden(dg.fb, self.kv)
            logits = self._full_logits(h, dg.fb)
            tok = samp_ops.sample(logits, temperature=st.temp, top_k=st.top_k, top_p=st.top_p,
                                  repetition_penalty=st.penalty, history=st.history,
                                  history_len=st.hist_len, seeds=st.seeds, offsets=st.offsets)
        # Device-side advance (one kernel) so back-to-back replays need no host round trip.
        ext().decode_advance(tok, dg.ids, dg.out, dg.meta, dg.valid, dg.block_table,
                             st.offsets if st is not None else None,
                             st.history if st is not None else None,
                             st.hist_len if st is not None else None)

    def graph_for(self, bsz: int, sampled: bool = False) -> DecodeGraph:
        dg = self.graphs.get((bsz, sampled))
        if dg is not None:
            return dg
        dg = self._make_graph(bsz, sampled)
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
        self.graphs[(bsz, sampled)] = dg
        return dg

    def replay(self, dg: DecodeGraph) -> None:
        if dg.graph is not None:
            dg.graph.replay()
        else:
            self._step_body(dg)

    def decode(self, ids: list[int], positions: list[int], pages: list[list[int]], *,
               sampling: list | None = None, history: list[list[int]] | None = None,
               steps: list[int] | None = None) -> list[int]:
        """Host-driven decode step: stage inputs (pinned H2D), replay, read tokens back.
        With ``sampling`` (SamplingParams or None per row) the sampling graph runs; ``steps``
        are the rows' token indices (Philox offsets) and ``history`` their prompt + output
        tokens (copied to the device only when the set of rows or their lengths changed)."""
        n = len(ids)
        dg = self.graph_for(bucket_for(n), sampled=sampling is not None)
        self.stage_decode_inputs(dg, ids, positions, pages)
        if sampling is not None:
            self._stage_sampling(dg, sampling, history or [[] for _ in ids], steps or [0] * n)
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

    def _stage_sampling(self, dg: DecodeGraph, sampling: list, history: list[list[int]],
                        steps: list[int]) -> None:
        st = dg.sampling
        n = len(sampling)
        t, k, p, r, sd = self._row_params(sampling)
        hf, hi, hk = st.host_f.numpy(), st.host_i.numpy(), st.host_k.numpy()
        hf[0, :] = 0.0
        hf[1, :] = 1.0
        hf[2, :] = 1.0
        hi[:] = 0
        hk[:] = 0
        hf[0, :n], hf[1, :n], hf[2, :n] = t, p, r
        hi[0, :n], hi[1, :n] = sd, steps
        hk[0, :n] = k
        lens = [len(x) for x in history]
        hk[1, :n] = lens
        key = (tuple(sd), tuple(lens))
        # The device appends each step's token itself; the history travels again only when
        # the rows changed (a new request, a finished one) since the last step.
        prev = st.key
        if prev is None or prev[0] != key[0] or tuple(x + 1 for x in prev[1]) != key[1]:
            hh = st.host_hist.numpy()
            hmax = hh.shape[1]
            for i, x in enumerate(history):
                m = min(len(x), hmax)
                hh[i, :m] = x[:m]
            st.history.copy_(st.host_hist, non_blocking=True)
        st.key = key
        st.temp.copy_(st.host_f[0], non_blocking=True)
        st.top_p.copy_(st.host_f[1], non_blocking=True)
        st.penalty.copy_(st.host_f[2], non_blocking=True)
        st.seeds.copy_(st.host_i[0], non_blocking=True)
        st.offsets.copy_(st.host_i[1], non_blocking=True)
        st.top_k.copy_(st.host_k[0], non_blocking=True)
        st.hist_len.copy_(st.host_k[1], non_blocking=True)
