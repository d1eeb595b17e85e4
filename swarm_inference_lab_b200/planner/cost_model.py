"""Plan cost model: predicted TTFT, decode rate and aggregate throughput, and the
objective score for the ``speed`` / ``throughput`` / ``capacity`` / ``balanced`` modes.

Every input is either measured or assumed; each assumed input multiplies the
score by ``unmeasured_penalty`` (0.98), so a measured plan wins a tie.

Reference: si/engines/cost_model.py:24-179 (PlanCostInputs, score_costs).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field


@dataclass
class PlanCostInputs:
    stage_compute_ms: list[float]          # per decode step, per stage
    boundary_ms: list[float]               # per decode step, per stage boundary
    prefill_ms: float                      # whole prompt
    batch: int = 1
    memory_fraction: float = 0.5           # max over workers of used / capacity
    unmeasured: list[str] = field(default_factory=list)
    replicas: int = 1


@dataclass
class PlanCosts:
    ttft_ms: float
    tpot_ms: float
    decode_tok_s: float
    aggregate_tok_s: float
    bottleneck_ms: float
    score: float
    mode: str


def score_costs(c: PlanCostInputs, mode: str = "balanced", unmeasured_penalty: float = 0.98) -> PlanCosts:
    # One token traverses every stage and boundary serially (no intra-request overlap);
    # with micro-batches in flight the bottleneck stage bounds throughput.
    tpot = sum(c.stage_compute_ms) + sum(c.boundary_ms)
    bottleneck = max(c.stage_compute_ms + (c.boundary_ms or [0.0]))
    decode = 1000.0 / tpot if tpot > 0 else 0.0
    stages = max(1, len(c.stage_compute_ms))
    pipelined = min(stages, c.batch)
    aggregate = c.replicas * c.batch * 1000.0 / max(bottleneck * pipelined, tpot) if tpot > 0 else 0.0
    ttft = c.prefill_ms + sum(c.boundary_ms)
    if mode == "speed":
        s = decode / (1.0 + ttft / 10000.0)
    elif mode == "throughput":
        s = aggregate
    elif mode == "capacity":
        s = (1.0 - c.memory_fraction) * 100.0 + math.log1p(aggregate)
    else:
        s = math.sqrt(max(decode, 1e-9) * max(aggregate, 1e-9)) / (1.0 + ttft / 20000.0)
    s *= unmeasured_penalty ** len(c.unmeasured)
    return PlanCosts(ttft, tpot, decode, aggregate, bottleneck, s, mode)
