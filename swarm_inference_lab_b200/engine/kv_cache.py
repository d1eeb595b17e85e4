"""Paged KV cache resident on the GPU of a stage owner.

Pages hold 64 tokens of one layer's K (and V) for every local KV head:
``k[layer] : [num_pages, Hkv, 64, 128]``.  A sequence owns an ordered list of
pages (its block-table row); pages are reference counted so a forked
sequence can share a prefix copy-on-write.

The reference keeps a static ``[B, Hkv, Smax, D]`` tensor per layer with
prepare/commit append, snapshot/restore/fork/rollback
(si/model/qwen3_cache.py:25-360); paging replaces the static slab so that
sequences of different lengths share one pool without fragmentation.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

PAGE = 64


class OutOfPages(RuntimeError):
    pass


class PageAllocator:
    """Free-list page allocator with reference counts (host side)."""

    def __init__(self, num_pages: int):
        self.num_pages = num_pages
        self._free = list(range(num_pages - 1, -1, -1))
        self._ref = [0] * num_pages

    @property
    def free(self) -> int:
        return len(self._free)

    def alloc(self, n: int) -> list[int]:
        if n > len(self._free):
            raise OutOfPages(f"need {n} pages, {len(self._free)} free")
        out = [self._free.pop() for _ in range(n)]
        for p in out:
            self._ref[p] = 1
        return out

    def retain(self, pages: list[int]) -> None:
        for p in pages:
            self._ref[p] += 1

    def release(self, pages: list[int]) -> None:
        for p in pages:
            self._ref[p] -= 1
            if self._ref[p] == 0:
                self._free.append(p)
            elif self._ref[p] < 0:
                raise RuntimeError(f"page {p} released twice")

    def refcount(self, p: int) -> int:
        return self._ref[p]


@dataclass
class SeqPages:
    pages: list[int] = field(default_factory=list)
    length: int = 0  # tokens stored


class PagedKVCache:
    def __init__(self, num_layers: int, num_kv_heads: int, num_pages: int, device,
                 head_dim: int = 128, dtype=torch.bfloat16, latent_dim: int | None = None):
        """``latent_dim`` set: one MLA latent row per token, ``k[layer] : [num_pages, 64,
        latent_dim]`` and no separate V (the latent cache holds both)."""
        self.num_layers = num_layers
        self.num_kv_heads = num_kv_heads
        self.num_pages = num_pages
        self.head_dim = head_dim
        self.latent_dim = latent_dim
        self.device = torch.device(device)
        if latent_dim is not None:
            self.k = torch.zeros((num_layers, num_pages, PAGE, latent_dim), dtype=dtype,
                                 device=self.device)
            self.v = None
        else:
            shape = (num_layers, num_pages, num_kv_heads, PAGE, head_dim)
            self.k = torch.zeros(shape, dtype=dtype, device=self.device)
            self.v = torch.zeros(shape, dtype=dtype, device=self.device)
        self.alloc = PageAllocator(num_pages)
        self.seqs: dict[str, SeqPages] = {}

    @staticmethod
    def pages_for(tokens: int) -> int:
        return (tokens + PAGE - 1) // PAGE

    @classmethod
    def bytes_per_page(cls, num_layers: int, num_kv_heads: int, head_dim: int = 128,
                       elem: int = 2) -> int:
        return 2 * num_layers * num_kv_heads * PAGE * head_dim * elem

    def layer(self, i: int):
        return self.k[i], (self.v[i] if self.v is not None else None)

    # ------------------------------------------------------------ sequences
    def open(self, seq_id: str) -> SeqPages:
        if seq_id in self.seqs:
            raise KeyError(f"sequence {seq_id} already open")
        s = SeqPages()
        self.seqs[seq_id] = s
        return s

    def reserve(self, seq_id: str, total_tokens: int) -> SeqPages:
        """Make sure the sequence owns pages for ``total_tokens`` tokens."""
        s = self.seqs[seq_id]
        need = self.pages_for(total_tokens) - len(s.pages)
        if need > 0:
            s.pages.extend(self.alloc.alloc(need))
        return s

    def slots(self, seq_id: str, start: int, count: int) -> list[int]:
        s = self.seqs[seq_id]
        return [s.pages[p // PAGE] * PAGE + p % PAGE for p in range(start, start + count)]

    def close(self, seq_id: str) -> None:
        s = self.seqs.pop(seq_id, None)
        if s is not None:
            self.alloc.release(s.pages)

    def fork(self, src: str, dst: str) -> None:
        """Share all of ``src``'s pages with a new sequence ``dst`` (prefix reuse)."""
        s = self.seqs[src]
        self.alloc.retain(s.pages)
        self.seqs[dst] = SeqPages(pages=list(s.pages), length=s.length)

    def truncate(self, seq_id: str, length: int) -> None:
        """Roll a sequence back to ``length`` tokens, releasing unused whole pages."""
        s = self.seqs[seq_id]
        keep = self.pages_for(length)
        if keep < len(s.pages):
            self.alloc.release(s.pages[keep:])
            del s.pages[keep:]
        s.length = min(s.length, length)

    def snapshot(self, seq_id: str) -> dict:
        """Host copy of the sequence's KV (checkpoint / migration payload)."""
        s = self.seqs[seq_id]
        idx = torch.tensor(s.pages, dtype=torch.long, device=self.device)
        return {"length": s.length, "k": self.k[:, idx].cpu(),
                "v": self.v[:, idx].cpu() if self.v is not None else None}

    def restore(self, seq_id: str, snap: dict) -> None:
        if seq_id not in self.seqs:
            self.open(seq_id)
        s = self.reserve(seq_id, max(1, int(snap["length"])))
        n = snap["k"].shape[1]
        idx = torch.tensor(s.pages[:n], dtype=torch.long, device=self.device)
        self.k[:, idx] = snap["k"].to(self.device)
        if self.v is not None:
            self.v[:, idx] = snap["v"].to(self.device)
        s.length = int(snap["length"])
