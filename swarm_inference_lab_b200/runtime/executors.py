"""Stage executors: the compute behind one persistent stage owner.

A stage executor owns a contiguous layer interval and per-session KV state.
Stage 0 takes token ids, later stages take hidden states ``[T, H]``; the last
stage returns logits of the new positions.  Two implementations:

* ``ReferenceStageExecutor`` - the PyTorch decoder (CPU fp32 for loopback
  pipelines and tests, or any device/dtype);
* ``KernelStageExecutor`` - the sm_100a kernels over a paged KV cache on one
  GPU (``models/dense.py``), for stage owners on B200s.

Interface after si/execution/interfaces.py:55 (``StageExecutor``) with the
session lifecycle of si/worker/stage_runtime.py:1391-2275.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Protocol

import torch

from ..models.config import ModelConfig
from ..models.reference import RefCache, ReferenceDecoder


@dataclass(frozen=True)
class StageSpec:
    stage_id: int
    layer_start: int
    layer_end: int
    num_stages: int

    @property
    def is_first(self) -> bool:
        return self.stage_id == 0

    @property
    def is_last(self) -> bool:
        return self.stage_id == self.num_stages - 1


class StageExecutor(Protocol):
    spec: StageSpec

    def open(self, session_id: str) -> None: ...

    def close(self, session_id: str) -> None: ...

    def forward(self, session_id: str, x: torch.Tensor, position: int) -> torch.Tensor: ...

    def length(self, session_id: str) -> int: ...

    def truncate(self, session_id: str, length: int) -> None: ...


class ReferenceStageExecutor:
    def __init__(self, cfg: ModelConfig, spec: StageSpec, get, *, device="cpu",
                 dtype=torch.float32):
        self.cfg = cfg
        self.spec = spec
        self.model = ReferenceDecoder(cfg, get, device=device, dtype=dtype,
                                      layer_range=(spec.layer_start, spec.layer_end),
                                      with_embed=spec.is_first, with_head=spec.is_last)
        self.sessions: dict[str, RefCache] = {}
        self.loads = 1  # weights are materialised once per owner

    def open(self, session_id: str) -> None:
        if session_id in self.sessions:
            raise KeyError(f"session {session_id} already open")
        self.sessions[session_id] = self.model.new_cache()

    def close(self, session_id: str) -> None:
        self.sessions.pop(session_id, None)

    def length(self, session_id: str) -> int:
        return self.sessions[session_id].length

    def truncate(self, session_id: str, length: int) -> None:
        self.sessions[session_id].truncate(length)

    @torch.no_grad()
    def forward(self, session_id: str, x: torch.Tensor, position: int) -> torch.Tensor:
        cache = self.sessions[session_id]
        if cache.length != position:
            raise ValueError(f"session {session_id}: cache holds {cache.length} tokens, "
                             f"frame is at position {position}")
        return self.model.forward(x, cache)


class KernelStageExecutor:
    """Paged-KV GPU stage on the sm_100a kernels (bf16)."""

    def __init__(self, cfg: ModelConfig, spec: StageSpec, get, *, device="cuda",
                 max_seq_len: int = 4096, kv_pages: int = 1024):
        from ..engine.kv_cache import PAGE, PagedKVCache
        from ..models.dense import DenseModel, DenseWeights, TPInfo
        self.cfg = cfg
        self.spec = spec
        self.device = torch.device(device)
        w = DenseWeights.from_full(cfg, TPInfo(), get, self.device,
                                   layer_range=(spec.layer_start, spec.layer_end),
                                   with_embed=spec.is_first, with_head=spec.is_last)
        self.model = DenseModel(w, self.device, max_positions=max_seq_len + PAGE)
        self.kv = PagedKVCache(self.model.num_layers, self.model.num_kv_local, kv_pages, self.device)
        self.max_pages = (max_seq_len + PAGE - 1) // PAGE
        self.page = PAGE

    def open(self, session_id: str) -> None:
        self.kv.open(session_id)

    def close(self, session_id: str) -> None:
        self.kv.close(session_id)

    def length(self, session_id: str) -> int:
        return self.kv.seqs[session_id].length

    def truncate(self, session_id: str, length: int) -> None:
        self.kv.truncate(session_id, length)

    @torch.no_grad()
    def forward(self, session_id: str, x: torch.Tensor, position: int) -> torch.Tensor:
        from ..models.dense import ForwardBatch
        seq = self.kv.seqs[session_id]
        if seq.length != position:
            raise ValueError(f"session {session_id}: cache holds {seq.length}, frame at {position}")
        T = x.shape[0]
        self.kv.reserve(session_id, position + T)
        dev = self.device
        pos = torch.arange(position, position + T, dtype=torch.int32)
        pages = torch.tensor(seq.pages, dtype=torch.int32)
        slots = pages[(pos // self.page).long()] * self.page + pos % self.page
        bt = torch.zeros((1, self.max_pages), dtype=torch.int32)
        bt[0, : len(seq.pages)] = pages
        fb = ForwardBatch(
            ids=x.to(dev).long() if self.spec.is_first else torch.zeros(T, dtype=torch.int64, device=dev),
            positions=pos.to(dev), slots=slots.to(dev),
            seq_lens=torch.tensor([position + T], dtype=torch.int32, device=dev),
            block_table=bt.to(dev), last_idx=torch.arange(T, device=dev), is_decode=False,
            cu_q=torch.tensor([0, T], dtype=torch.int32, device=dev), max_q_len=T)
        h = None if self.spec.is_first else x.to(dev, torch.bfloat16).contiguous()
        h = self.model.forward_hidden(fb, self.kv, h=h)
        seq.length = position + T
        if self.spec.is_last:
            return self.model.logits(h, fb)
        return h
