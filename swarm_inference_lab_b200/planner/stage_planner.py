"""Cross-host pipeline planner: bounded, deterministic beam search over contiguous
N-stage plans on heterogeneous workers connected by measured links.

A plan is an ordered list of (worker, layer interval).  The beam grows plans
stage by stage; each partial plan is scored by the cost model with measured
per-worker decode rates and per-link transfer times (boundary activation
bytes + token return), and only ``beam_width`` states survive each step.
Memory caps prune infeasible intervals; ties break on a canonical key so
the result is deterministic.  Limits: beam 512, <= 32 stages, <= 64 workers.

Reference: si/coordinator/stage_planner.py:181-1099 (_beam_key, build_plan,
_evaluate_candidate, _network_ms).
"""
from __future__ import annotations

from dataclasses import dataclass, field

from .cost_model import PlanCostInputs, PlanCosts, score_costs
from .topology import LinkProfile, transfer_ms


@dataclass(frozen=True)
class WorkerCaps:
    worker_id: str
    layer_ms: float            # measured decode time of one layer at the planned batch
    memory_bytes: float
    measured: bool = True


@dataclass
class StagePlan:
    stages: list[tuple[str, int, int]]
    costs: PlanCosts
    explain: dict = field(default_factory=dict)


class PlanningError(RuntimeError):
    pass


def build_plan(num_layers: int, layer_bytes: float, embed_bytes: float, head_bytes: float,
               workers: list[WorkerCaps], links: dict[tuple[str, str], LinkProfile], *,
               boundary_bytes: int, prompt_tokens: int = 512, batch: int = 1,
               mode: str = "balanced", beam_width: int = 512, max_stages: int = 32,
               coordinator: str = "coordinator") -> StagePlan:
    if not workers:
        raise PlanningError("no workers")
    if len(workers) > 64:
        raise PlanningError("at most 64 workers")
    wmap = {w.worker_id: w for w in workers}

    def link_ms(a, b, nbytes):
        lk = links.get((a, b))
        return transfer_ms(lk, nbytes) if lk else 50.0 + nbytes / 12.5e6 * 1e3

    # state: (layers_done, used_workers(tuple), stages(list))
    beam: list[tuple[int, tuple, list]] = [(0, (), [])]
    finished: list[StagePlan] = []
    for _ in range(min(max_stages, len(workers))):
        nxt = []
        for done, used, stages in beam:
            for w in workers:
                if w.worker_id in used:
                    continue
                for end in range(done + 1, num_layers + 1):
                    mem = (end - done) * layer_bytes + (embed_bytes if done == 0 else 0) + \
                          (head_bytes if end == num_layers else 0)
                    if mem > w.memory_bytes:
                        break
                    st = stages + [(w.worker_id, done, end)]
                    if end == num_layers:
                        finished.append(_evaluate(st, wmap, link_ms, boundary_bytes, prompt_tokens,
                                                  batch, mode, coordinator))
                    else:
                        nxt.append((end, used + (w.worker_id,), st))
        if not nxt:
            break

        def key(s):
            done, used, stages = s
            partial = sum((e - b) * wmap[wid].layer_ms for wid, b, e in stages)
            return (-done / max(partial, 1e-9), tuple(stages))
        nxt.sort(key=key)
        beam = nxt[:beam_width]
    if not finished:
        raise PlanningError("no worker combination holds the model")
    finished.sort(key=lambda p: (-p.costs.score, [s for s in p.stages]))
    return finished[0]


def _evaluate(stages, wmap, link_ms, boundary_bytes, prompt_tokens, batch, mode, coordinator):
    compute = [(e - b) * wmap[w].layer_ms for w, b, e in stages]
    bounds = [link_ms(stages[i][0], stages[i + 1][0], boundary_bytes * batch)
              for i in range(len(stages) - 1)]
    # token returns to stage 0 and the coordinator publication
    bounds.append(link_ms(stages[-1][0], stages[0][0], 8 * batch))
    prefill = sum(c * prompt_tokens / 8 for c in compute) + \
        sum(link_ms(stages[i][0], stages[i + 1][0], boundary_bytes * prompt_tokens)
            for i in range(len(stages) - 1))
    unmeasured = [w for w, _, _ in stages if not wmap[w].measured]
    costs = score_costs(PlanCostInputs(compute, bounds, prefill, batch=batch, unmeasured=unmeasured), mode)
    return StagePlan(list(stages), costs, {"compute_ms": compute, "boundary_ms": bounds,
                                           "prefill_ms": prefill})
