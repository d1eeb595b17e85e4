"""Deterministic discrete-event simulation of a stage ring and of an expert-parallel layer.

* ``Simulator``: a seeded event queue with a simulated clock (no wall time).
* ``Link``: latency + bytes / bandwidth, seeded jitter, loss and payload corruption
  (corrupted frames are detected by their checksum and resent, as the stage ring does).
* ``StageNode``: a FIFO server with a per-token service time; a node can fail and
  recover (churn); requests in flight on a failed node are replayed from the last
  accepted token (restart-and-replay), costing the replay prefill.
* ``simulate_ring``: requests flow stage 0 -> ... -> last -> back to the coordinator,
  one token per round trip; returns per-request TTFT / TPOT and aggregate tokens/s.
* ``expert_layer_time``: time of one EP MoE layer given per-expert token counts,
  expert compute rate and the dispatch / combine bytes over the links (the slowest
  rank sets the layer time), used to study load imbalance.

Reference: si/simulation/simulator.py:129, si/simulation/network.py:33,98,
si/simulation/expert_model.py:36,163.
"""
from __future__ import annotations

import heapq
import itertools
import random
import statistics
from dataclasses import dataclass, field


class Simulator:
    def __init__(self, seed: int = 0):
        self.now = 0.0
        self.rng = random.Random(seed)
        self._q: list = []
        self._ids = itertools.count()

    def at(self, t: float, fn, *args) -> None:
        heapq.heappush(self._q, (max(t, self.now), next(self._ids), fn, args))

    def after(self, dt: float, fn, *args) -> None:
        self.at(self.now + max(0.0, dt), fn, *args)

    def run(self, until: float = float("inf"), max_events: int = 10_000_000) -> int:
        n = 0
        while self._q and n < max_events:
            t, _, fn, args = self._q[0]
            if t > until:
                break
            heapq.heappop(self._q)
            self.now = t
            fn(*args)
            n += 1
        return n


@dataclass
class Link:
    latency_s: float = 100e-6
    bandwidth_Bps: float = 10e9
    jitter_s: float = 0.0
    loss: float = 0.0
    corruption: float = 0.0
    resends: int = 0

    def delay(self, sim: Simulator, nbytes: int) -> float:
        t = 0.0
        while True:
            j = sim.rng.uniform(-self.jitter_s, self.jitter_s) if self.jitter_s else 0.0
            t += max(0.0, self.latency_s + j) + nbytes / self.bandwidth_Bps
            bad = (self.loss and sim.rng.random() < self.loss) or \
                  (self.corruption and sim.rng.random() < self.corruption)
            if not bad:
                return t
            self.resends += 1          # lost or checksum failure: resend after a timeout-free NACK


@dataclass
class StageNode:
    name: str
    decode_s: float                  # service time of one decode token
    prefill_s_per_token: float
    up: bool = True
    busy_until: float = 0.0
    failures: list = field(default_factory=list)

    def service(self, sim: Simulator, tokens: int, prefill: bool) -> float:
        start = max(sim.now, self.busy_until)
        dur = tokens * self.prefill_s_per_token if prefill else self.decode_s
        self.busy_until = start + dur
        return self.busy_until - sim.now


@dataclass
class RequestTrace:
    rid: int
    prompt: int
    tokens: int
    start: float = 0.0
    first: float | None = None
    done: float | None = None
    emitted: int = 0
    replays: int = 0


def simulate_ring(stages: list[StageNode], link: Link, *, requests: int, prompt_tokens: int,
                  output_tokens: int, hidden_bytes: int, arrival_s: float = 0.0,
                  churn: list[tuple[float, int, float]] = (), seed: int = 0) -> dict:
    """``churn``: (time, stage index, downtime) failures.  Returns latency / throughput stats."""
    sim = Simulator(seed)
    traces = [RequestTrace(i, prompt_tokens, output_tokens) for i in range(requests)]

    def fail(si: int, down: float):
        stages[si].up = False
        stages[si].failures.append(sim.now)
        sim.after(down, recover, si)

    def recover(si: int):
        stages[si].up = True

    for t, si, down in churn:
        sim.at(t, fail, si, down)

    def hop(tr: RequestTrace, si: int, prefill: bool, tokens: int):
        node = stages[si]
        if not node.up:
            # restart-and-replay: wait for the node, then rebuild the context from the log
            tr.replays += 1
            sim.after(0.01, hop, tr, si, True, tr.prompt + tr.emitted)
            return
        dt = node.service(sim, tokens, prefill)
        nbytes = hidden_bytes * (tokens if prefill else 1)
        if si + 1 < len(stages):
            sim.after(dt + link.delay(sim, nbytes), hop, tr, si + 1, prefill, tokens)
        else:
            sim.after(dt + link.delay(sim, 64), token_back, tr)

    def token_back(tr: RequestTrace):
        tr.emitted += 1
        if tr.first is None:
            tr.first = sim.now
        if tr.emitted >= tr.tokens:
            tr.done = sim.now
            return
        hop(tr, 0, False, 1)

    def start(tr: RequestTrace):
        tr.start = sim.now
        hop(tr, 0, True, tr.prompt)

    for i, tr in enumerate(traces):
        sim.at(i * arrival_s, start, tr)
    sim.run()
    done = [t for t in traces if t.done is not None]
    span = max(t.done for t in done) - min(t.start for t in done) if done else 0.0
    ttft = [t.first - t.start for t in done]
    tpot = [(t.done - t.first) / max(1, t.tokens - 1) for t in done]
    return {"completed": len(done), "tokens_per_s": sum(t.emitted for t in done) / span if span else 0.0,
            "ttft_p50_s": statistics.median(ttft) if ttft else None,
            "tpot_p50_s": statistics.median(tpot) if tpot else None,
            "replays": sum(t.replays for t in traces), "resends": link.resends,
            "sim_time_s": sim.now}


def expert_layer_time(tokens_per_expert: list[int], owner: list[int], ranks: int, *,
                      flops_per_token: float, rate_flops: float, weight_bytes_per_expert: float,
                      hbm_Bps: float, token_bytes: float, link_Bps: float, link_latency_s: float) -> dict:
    """One EP layer: each rank streams the weights of its touched experts and computes its
    tokens; dispatch / combine move token rows over the links.  The slowest rank wins."""
    per_rank = []
    for r in range(ranks):
        mine = [i for i, o in enumerate(owner) if o == r]
        toks = sum(tokens_per_expert[i] for i in mine)
        touched = sum(1 for i in mine if tokens_per_expert[i] > 0)
        compute = max(toks * flops_per_token / rate_flops, touched * weight_bytes_per_expert / hbm_Bps)
        comm = 2 * (link_latency_s + toks * token_bytes / link_Bps)
        per_rank.append(compute + comm)
    mean = statistics.fmean(per_rank)
    return {"layer_s": max(per_rank), "imbalance": max(per_rank) / mean if mean else 1.0,
            "per_rank_s": per_rank}


def zipf_tokens(experts: int, tokens: int, top_k: int, skew: float, seed: int = 0) -> list[int]:
    """Token counts per expert for ``tokens`` x ``top_k`` routed assignments with Zipf skew."""
    rng = random.Random(seed)
    w = [1.0 / (i + 1) ** skew for i in range(experts)]
    counts = [0] * experts
    idx = list(range(experts))
    for _ in range(tokens):
        chosen = set()
        while len(chosen) < top_k:
            chosen.add(rng.choices(idx, weights=w)[0])
        for e in chosen:
            counts[e] += 1
    return counts
