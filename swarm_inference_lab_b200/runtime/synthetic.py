"""Deterministic, calibrated synthetic stages.

A synthetic stage stands in for a real layer interval when a test or the simulator
needs stage owners without weights: it maps ``[T, H]`` activations (or token ids on
the first stage) through a fixed, cheap, invertible-looking transform seeded by
(stage id, layer range) and sleeps (busy-waits) for a calibrated time per token so
that loopback rings reproduce a target per-stage latency.  The last stage derives a
token id from a hash of its activations, so a ring of synthetic stages produces a
deterministic token stream that depends on every stage's output.

Reference: si/model/synthetic.py:25 ``deterministic_cpu_kernel``, :78.
"""
from __future__ import annotations

import hashlib
import time
from dataclasses import dataclass

import torch

from .executors import StageSpec


@dataclass
class SyntheticCalibration:
    prefill_s_per_token: float = 0.0
    decode_s: float = 0.0


def deterministic_kernel(x: torch.Tensor, seed: int) -> torch.Tensor:
    """Elementwise mix with per-column constants derived from ``seed`` (fp32, CPU)."""
    g = torch.Generator().manual_seed(seed)
    H = x.shape[-1]
    a = torch.rand(H, generator=g) * 0.5 + 0.75
    b = torch.randn(H, generator=g) * 0.01
    return torch.tanh(x.float() * a + b)


class SyntheticStageExecutor:
    def __init__(self, spec: StageSpec, hidden: int, vocab: int, *,
                 calib: SyntheticCalibration | None = None, seed: int = 0):
        self.spec = spec
        self.hidden = hidden
        self.vocab = vocab
        self.calib = calib or SyntheticCalibration()
        self.seed = seed * 1_000_003 + spec.stage_id * 7919 + spec.layer_start
        self.lengths: dict[str, int] = {}

    def open(self, session_id: str) -> None:
        self.lengths[session_id] = 0

    def close(self, session_id: str) -> None:
        self.lengths.pop(session_id, None)

    def length(self, session_id: str) -> int:
        return self.lengths[session_id]

    def truncate(self, session_id: str, length: int) -> None:
        self.lengths[session_id] = min(self.lengths[session_id], length)

    def _busy(self, seconds: float) -> None:
        end = time.perf_counter() + seconds
        while time.perf_counter() < end:
            pass

    def forward(self, session_id: str, x: torch.Tensor, position: int) -> torch.Tensor:
        T = x.shape[0]
        self._busy(self.calib.decode_s if T == 1 else T * self.calib.prefill_s_per_token)
        if self.spec.is_first:
            ids = x.long().view(-1)
            h = torch.stack([deterministic_kernel(torch.full((self.hidden,), float(i % 997) / 997.0),
                                                  self.seed + p)
                             for p, i in enumerate(ids.tolist(), start=position)])
        else:
            h = deterministic_kernel(x, self.seed)
        self.lengths[session_id] = position + T
        if self.spec.is_last:
            tok = []
            for row in h:
                d = hashlib.sha256(row.numpy().tobytes()).digest()
                tok.append(int.from_bytes(d[:4], "little") % self.vocab)
            return torch.tensor(tok, dtype=torch.int64)
        return h


def calibrate(target_decode_ms: float, target_prefill_ms_per_token: float) -> SyntheticCalibration:
    return SyntheticCalibration(target_prefill_ms_per_token / 1e3, target_decode_ms / 1e3)
