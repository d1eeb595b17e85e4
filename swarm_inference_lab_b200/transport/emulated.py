"""Deterministic emulated transport with a simulated clock.

Wraps a request handler (the same ``async handler(msg) -> list[msg]`` a stage
server uses) behind a link model: each request costs ``latency_s + bytes /
bandwidth`` of simulated time on the link, with optional seeded jitter and drop
probability.  Time advances only through ``SimClock``, so runs are exactly
reproducible and take no wall time; the simulator and planner tests drive
multi-stage rings through it.

Reference: si/transport/emulated_transport.py:23.
"""
from __future__ import annotations

import random
from dataclasses import dataclass


class SimClock:
    def __init__(self):
        self.now = 0.0

    def advance(self, dt: float) -> float:
        self.now += max(0.0, dt)
        return self.now


class LinkDropped(ConnectionError):
    pass


@dataclass
class LinkModel:
    latency_s: float = 50e-6
    bandwidth_Bps: float = 25e9
    jitter_s: float = 0.0
    drop_prob: float = 0.0

    def cost(self, nbytes: int, rng: random.Random) -> float:
        j = rng.uniform(-self.jitter_s, self.jitter_s) if self.jitter_s else 0.0
        return max(0.0, self.latency_s + j) + nbytes / self.bandwidth_Bps


class EmulatedTransport:
    def __init__(self, handler, link: LinkModel, clock: SimClock | None = None, seed: int = 0):
        self.handler = handler
        self.link = link
        self.clock = clock or SimClock()
        self.rng = random.Random(seed)
        self.sent_bytes = 0
        self.requests = 0

    async def request(self, msg, nbytes: int | None = None):
        from ..protocol import stage_ring as sr
        size = nbytes if nbytes is not None else len(sr.encode(msg))
        self.requests += 1
        if self.link.drop_prob and self.rng.random() < self.link.drop_prob:
            self.clock.advance(self.link.latency_s)
            raise LinkDropped("emulated link dropped the frame")
        self.clock.advance(self.link.cost(size, self.rng))
        self.sent_bytes += size
        replies = await self.handler(msg)
        for r in replies or []:
            rb = len(sr.encode(r))
            self.sent_bytes += rb
            self.clock.advance(self.link.cost(rb, self.rng))
        return replies
