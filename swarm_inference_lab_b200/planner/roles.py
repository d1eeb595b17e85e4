"""Heterogeneous node roles by marginal utility.

Nodes are considered in descending capability; each is assigned the role
with the largest marginal gain in aggregate tokens/s (``stage`` owner in a
pipeline replica, ``expert`` host, ``draft`` model host, or ``idle`` when
nothing helps - a node that would slow the plan down is left idle).

Reference: si/planner.py:16-424 (heterogeneous role planner).
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class NodeCaps:
    node_id: str
    decode_tok_s: float        # measured single-node decode rate for the model shard it can hold
    memory_bytes: float
    link_ms: float             # one-way latency to the fastest peer


@dataclass
class RoleAssignment:
    node_id: str
    role: str
    gain_tok_s: float


def assign_roles(nodes: list[NodeCaps], model_bytes: float, *, expert_fraction: float = 0.0
                 ) -> list[RoleAssignment]:
    out = []
    pipeline_rate = 0.0
    pipeline_mem = 0.0
    members = 0
    for n in sorted(nodes, key=lambda n: (-n.decode_tok_s, n.node_id)):
        # joining the pipeline: its rate is bounded by the slowest member, but memory adds up
        if pipeline_mem < model_bytes:
            new_mem = pipeline_mem + n.memory_bytes
            gain = (min(pipeline_rate or n.decode_tok_s, n.decode_tok_s) if new_mem >= model_bytes else 0.0)
            out.append(RoleAssignment(n.node_id, "stage", gain))
            pipeline_mem = new_mem
            pipeline_rate = min(pipeline_rate or n.decode_tok_s, n.decode_tok_s)
            members += 1
            continue
        # the model is already held: extra nodes can host experts (MoE) or a replica
        replica_gain = n.decode_tok_s if n.memory_bytes >= model_bytes else 0.0
        expert_gain = expert_fraction * pipeline_rate * (1.0 / (1.0 + n.link_ms))
        latency_cost = pipeline_rate * n.link_ms / 100.0
        gain, role = max(((replica_gain, "replica"), (expert_gain - latency_cost, "expert")),
                         key=lambda o: o[0])
        if gain <= 0.0:              # nothing it could do adds tokens/s
            gain, role = 0.0, "idle"
        out.append(RoleAssignment(n.node_id, role, gain))
    return out
