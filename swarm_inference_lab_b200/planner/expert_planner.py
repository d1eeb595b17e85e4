"""Per-expert placement by measured utility: local, whole-remote, microshard-remote or hybrid.

For each expert the planner compares the expected milliseconds per decode
step of running it locally (if it fits the local budget), sending its rows
to one remote owner (link transfer both ways + remote compute), or
splitting its intermediate dimension across several microshard owners
(fan-out transfer + the slowest shard + a fixed-order reduction).
Experts are processed in descending activation frequency, so hot experts
claim local memory first.

Reference: si/coordinator/expert_planner.py:14-402.
"""
from __future__ import annotations

from dataclasses import dataclass

from .topology import LinkProfile, transfer_ms


@dataclass(frozen=True)
class ExpertStats:
    layer: int
    expert: int
    frequency: float            # expected tokens routed per decode step
    bytes: int


@dataclass(frozen=True)
class RemoteOwner:
    worker_id: str
    link: LinkProfile
    rows_per_ms: float          # measured expert throughput (tokens per ms)
    free_bytes: int


@dataclass
class ExpertDecision:
    layer: int
    expert: int
    placement: str              # local | whole_remote | microshard | hybrid
    owners: tuple[str, ...]
    expected_ms: float


def plan_experts(experts: list[ExpertStats], *, local_budget: int, local_rows_per_ms: float,
                 remotes: list[RemoteOwner], hidden: int, max_fanout: int = 4,
                 act_bytes: int = 2) -> list[ExpertDecision]:
    out = []
    budget = local_budget
    free = {r.worker_id: r.free_bytes for r in remotes}
    for e in sorted(experts, key=lambda x: (-x.frequency, x.layer, x.expert)):
        rows = max(e.frequency, 1e-6)
        row_bytes = hidden * act_bytes
        options = []
        if e.bytes <= budget:
            options.append((rows / local_rows_per_ms, "local", ()))
        for r in remotes:
            if free[r.worker_id] >= e.bytes:
                t = 2 * transfer_ms(r.link, int(rows * row_bytes)) + rows / r.rows_per_ms
                options.append((t, "whole_remote", (r.worker_id,)))
        cands = sorted((r for r in remotes if free[r.worker_id] >= e.bytes // max_fanout),
                       key=lambda r: transfer_ms(r.link, int(rows * row_bytes)))[:max_fanout]
        if len(cands) >= 2:
            k = len(cands)
            t = max(2 * transfer_ms(r.link, int(rows * row_bytes)) + rows / (r.rows_per_ms * k)
                    for r in cands) + 0.01 * k
            options.append((t, "microshard", tuple(r.worker_id for r in cands)))
        if not options:
            raise RuntimeError(f"expert {e.layer}/{e.expert} fits nowhere")
        t, kind, owners = min(options, key=lambda o: (o[0], o[1]))
        if kind == "local":
            budget -= e.bytes
        elif kind == "whole_remote":
            free[owners[0]] -= e.bytes
        else:
            for w in owners:
                free[w] -= e.bytes // len(owners)
        out.append(ExpertDecision(e.layer, e.expert, kind, owners, t))
    kinds = {d.placement for d in out}
    if len(kinds) > 1:
        for d in out:
            d.placement = d.placement if d.placement != "local" else "local"
    return out


def summarize(decisions: list[ExpertDecision]) -> dict:
    s: dict[str, int] = {}
    for d in decisions:
        s[d.placement] = s.get(d.placement, 0) + 1
    s["expected_ms"] = round(sum(d.expected_ms for d in decisions), 4)
    s["hybrid"] = len({d.placement for d in decisions}) > 1
    return s
