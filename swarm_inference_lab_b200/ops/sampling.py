"""Token selection on the device: greedy argmax (lowest id on ties)."""
from __future__ import annotations

import torch

from ._ext import ext


def argmax(logits: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    if out is None:
        out = torch.empty(logits.shape[0], dtype=torch.int64, device=logits.device)
    ext().argmax(logits, out)
    return out


def sample(logits: torch.Tensor, *, temperature, top_k=0, top_p=1.0, repetition_penalty=1.0,
           history: torch.Tensor | None = None, history_len: torch.Tensor | None = None,
           seeds=0, offsets=0, out: torch.Tensor | None = None) -> torch.Tensor:
    """Per-row sampling.  Scalars broadcast over rows; ``logits`` is modified in place by the
    repetition penalty.  temperature 0 = greedy (lowest id on ties)."""
    B = logits.shape[0]
    dev = logits.device

    def vec(x, dtype):
        if isinstance(x, torch.Tensor):
            return x.to(device=dev, dtype=dtype).reshape(B).contiguous()
        return torch.full((B,), x, dtype=dtype, device=dev)

    if out is None:
        out = torch.empty(B, dtype=torch.int64, device=dev)
    ext().sample_tokens(logits, vec(temperature, torch.float32), vec(top_k, torch.int32),
                        vec(top_p, torch.float32), vec(repetition_penalty, torch.float32),
                        history, history_len, vec(seeds, torch.int64), vec(offsets, torch.int64), out)
    return out


def sample_reference_probs(logits: torch.Tensor, temperature: float, top_k: int = 0,
                           top_p: float = 1.0) -> torch.Tensor:
    """The distribution ``sample`` draws from, in plain PyTorch (fp32)."""
    z = logits.float() / temperature
    if top_k > 0:
        kth = torch.topk(z, top_k, dim=-1).values[..., -1:]
        z = z.masked_fill(z < kth, float("-inf"))
    p = torch.softmax(z, dim=-1)
    if top_p < 1.0:
        sp, idx = torch.sort(p, dim=-1, descending=True)
        cum = sp.cumsum(-1)
        keep = (cum - sp) < top_p * p.sum(-1, keepdim=True)
        mask = torch.zeros_like(p, dtype=torch.bool).scatter(-1, idx, keep)
        p = torch.where(mask, p, torch.zeros_like(p))
        p = p / p.sum(-1, keepdim=True)
    return p


def embedding(ids: torch.Tensor, table: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    if out is None:
        out = torch.empty((ids.numel(), table.shape[1]), dtype=table.dtype, device=table.device)
    ext().embedding(ids, table, out)
    return out
