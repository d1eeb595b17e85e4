"""Topology-scoped stage session registry.

A stage owner keeps one record per open session: the topology and route
generation it was opened under, the KV position it has reached, the sequence's
pages in the resident cache, and timestamps.  Records are invalidated when the
route generation changes (a new deployment fences the old sessions), expire
after an idle TTL, and are bounded in number (least recently used first).

Reference: si/worker/stage_sessions.py:27.
"""
from __future__ import annotations

import time
from collections import OrderedDict
from dataclasses import dataclass, field


class SessionLimit(RuntimeError):
    pass


@dataclass
class StageSession:
    session_id: str
    topology_id: str
    generation: int
    position: int = 0
    pages: list[int] = field(default_factory=list)
    opened_at: float = field(default_factory=time.time)
    last_used: float = field(default_factory=time.time)


class StageSessionRegistry:
    def __init__(self, *, max_sessions: int = 4096, idle_ttl_s: float = 600.0):
        self.max = max_sessions
        self.ttl = idle_ttl_s
        self._s: OrderedDict[str, StageSession] = OrderedDict()

    def __len__(self) -> int:
        return len(self._s)

    def open(self, session_id: str, topology_id: str, generation: int, *, now: float | None = None,
             evict=None) -> StageSession:
        now = time.time() if now is None else now
        if session_id in self._s:
            raise KeyError(f"session {session_id} already open")
        self.expire(now=now, evict=evict)
        if len(self._s) >= self.max:
            old_id, old = self._s.popitem(last=False)
            if evict:
                evict(old)
        s = StageSession(session_id, topology_id, generation, opened_at=now, last_used=now)
        self._s[session_id] = s
        return s

    def get(self, session_id: str, *, topology_id: str, generation: int,
            now: float | None = None) -> StageSession:
        s = self._s.get(session_id)
        if s is None:
            raise KeyError(f"unknown session {session_id}")
        if s.topology_id != topology_id or s.generation != generation:
            raise KeyError(f"session {session_id} belongs to {s.topology_id}@{s.generation}")
        s.last_used = time.time() if now is None else now
        self._s.move_to_end(session_id)
        return s

    def advance(self, session_id: str, new_position: int) -> None:
        s = self._s[session_id]
        if new_position < s.position:
            raise ValueError("session positions only move forward (use truncate)")
        s.position = new_position

    def truncate(self, session_id: str, position: int) -> None:
        s = self._s[session_id]
        s.position = min(s.position, position)

    def close(self, session_id: str) -> StageSession | None:
        return self._s.pop(session_id, None)

    def invalidate_generation(self, generation: int, evict=None) -> list[str]:
        """Drop every session opened under an older route generation."""
        gone = [k for k, v in self._s.items() if v.generation < generation]
        for k in gone:
            s = self._s.pop(k)
            if evict:
                evict(s)
        return gone

    def expire(self, *, now: float | None = None, evict=None) -> list[str]:
        now = time.time() if now is None else now
        gone = [k for k, v in self._s.items() if now - v.last_used > self.ttl]
        for k in gone:
            s = self._s.pop(k)
            if evict:
                evict(s)
        return gone

    def snapshot(self) -> list[dict]:
        return [dict(s.__dict__) for s in self._s.values()]
