"""Token selection on the device: greedy argmax (lowest id on ties)."""
from __future__ import annotations

import torch

from ._ext import ext


def argmax(logits: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    if out is None:
        out = torch.empty(logits.shape[0], dtype=torch.int64, device=logits.device)
    ext().argmax(logits, out)
    return out


def embedding(ids: torch.Tensor, table: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    if out is None:
        out = torch.empty((ids.numel(), table.shape[1]), dtype=table.dtype, device=table.device)
    ext().embedding(ids, table, out)
    return out
