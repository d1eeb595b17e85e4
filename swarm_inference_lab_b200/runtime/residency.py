"""Tensor residency tracker visible to the planner.

Records where each named tensor lives (``device:N``, ``host_pinned``, ``host``,
``disk``), its size, and every movement between tiers with its byte count and
duration, plus hit/miss counts of lookups (a hit is a lookup that found the tensor
already on the requested tier).  The planner reads ``bytes_on`` / ``moved_bytes`` /
``hit_rate`` to cost plans that would page experts or KV between HBM and host.

Reference: si/runtime/residency.py:82.
"""
from __future__ import annotations

import time
from collections import defaultdict
from dataclasses import dataclass, field


@dataclass
class Residency:
    name: str
    tier: str
    nbytes: int
    pinned: bool = False
    last_access: float = field(default_factory=time.time)


@dataclass
class Movement:
    name: str
    src: str
    dst: str
    nbytes: int
    seconds: float
    at: float


class ResidencyTracker:
    def __init__(self):
        self.tensors: dict[str, Residency] = {}
        self.moves: list[Movement] = []
        self.hits = 0
        self.misses = 0

    def place(self, name: str, tier: str, nbytes: int, *, pinned: bool = False) -> None:
        self.tensors[name] = Residency(name, tier, int(nbytes), pinned)

    def lookup(self, name: str, tier: str) -> bool:
        r = self.tensors.get(name)
        ok = r is not None and r.tier == tier
        if ok:
            self.hits += 1
            r.last_access = time.time()
        else:
            self.misses += 1
        return ok

    def move(self, name: str, dst: str, seconds: float = 0.0) -> Movement:
        r = self.tensors[name]
        if r.pinned and dst != r.tier:
            raise ValueError(f"{name} is pinned to {r.tier}")
        m = Movement(name, r.tier, dst, r.nbytes, seconds, time.time())
        r.tier = dst
        r.last_access = m.at
        self.moves.append(m)
        return m

    def evict_candidates(self, tier: str, need_bytes: int) -> list[str]:
        """Least recently used unpinned tensors on ``tier`` covering ``need_bytes``."""
        out, got = [], 0
        for r in sorted((r for r in self.tensors.values() if r.tier == tier and not r.pinned),
                        key=lambda r: r.last_access):
            if got >= need_bytes:
                break
            out.append(r.name)
            got += r.nbytes
        return out

    def bytes_on(self) -> dict[str, int]:
        d: dict[str, int] = defaultdict(int)
        for r in self.tensors.values():
            d[r.tier] += r.nbytes
        return dict(d)

    def moved_bytes(self, src: str | None = None, dst: str | None = None) -> int:
        return sum(m.nbytes for m in self.moves if (src is None or m.src == src)
                   and (dst is None or m.dst == dst))

    def hit_rate(self) -> float:
        n = self.hits + self.misses
        return self.hits / n if n else 1.0

    def summary(self) -> dict:
        return {"bytes_on": self.bytes_on(), "moves": len(self.moves),
                "moved_bytes": self.moved_bytes(), "hit_rate": round(self.hit_rate(), 4)}
