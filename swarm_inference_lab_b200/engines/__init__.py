"""Execution engines, their capability probes and plan competition.

* ``ExecutionEngine`` protocol: ``probe(capabilities) -> EngineSupportReport``,
  ``candidate_plans(model, capabilities, request) -> [ExecutionPlan]``.
* ``NativeStageEngine``: this runtime's sm_100a stage owners - on one NVLink
  box it asks the box planner for TP/EP/PP splits; across hosts it asks the
  stage planner for a contiguous pipeline.
* ``ExternalEngineSlot``: registry entries for engines the reference could
  delegate to (llama.cpp RPC, SGLang, Colibri).  They probe "unavailable" on
  a B200 box without those binaries and never win a competition here.
* ``EngineRegistry.compete``: probe all engines, collect candidate plans,
  apply network competition factors (measurement confidence x1 / 0.96 /
  0.88, and 0.94 per WAN boundary) and the mechanism policy gates, and
  return the best admissible plan with every rejection recorded.

Reference: si/engines/interfaces.py:45-742, si/engines/registry.py:28-226,
si/engines/native_stage.py:126-826, si/coordinator/canonical_planner.py:21-267.
"""
from __future__ import annotations

import enum
import shutil
from dataclasses import dataclass, field
from typing import Protocol

from ..models.config import ModelConfig
from ..planner.box_planner import BoxMeasurements, plan_box
from ..planner.topology import Domain


class Policy(str, enum.Enum):
    REQUIRED = "required"
    AVAILABLE_CONDITIONAL = "available_conditional"
    REJECTED_DEFAULT = "rejected_default"
    EVIDENCE_ONLY = "evidence_only"


@dataclass
class ClusterCapabilities:
    nodes: dict[str, dict] = field(default_factory=dict)       # node -> {gpus, gpu_name, memory_gb}
    links: dict[tuple[str, str], Domain] = field(default_factory=dict)
    measurements: BoxMeasurements = field(default_factory=BoxMeasurements)
    measured_links: bool = True

    @property
    def total_gpus(self) -> int:
        return sum(int(n.get("gpus", 0)) for n in self.nodes.values())


@dataclass
class EngineSupportReport:
    engine: str
    available: bool
    reasons: list[str] = field(default_factory=list)


@dataclass
class ExecutionPlan:
    engine: str
    description: str
    parallelism: dict
    predicted_tok_s: float
    predicted_ttft_ms: float
    predicted_tpot_ms: float
    score: float
    mechanisms: list[str] = field(default_factory=list)
    wan_boundaries: int = 0
    confidence: str = "measured"   # measured | partial | assumed
    explain: dict = field(default_factory=dict)


@dataclass
class RequestShape:
    batch: int = 1
    prompt_tokens: int = 512
    output_tokens: int = 128
    mode: str = "balanced"
    require_distributed: bool = False


class ExecutionEngine(Protocol):
    name: str

    def probe(self, caps: ClusterCapabilities) -> EngineSupportReport: ...

    def candidate_plans(self, cfg: ModelConfig, caps: ClusterCapabilities,
                        req: RequestShape) -> list[ExecutionPlan]: ...


class NativeStageEngine:
    name = "native-stage"

    def probe(self, caps):
        reasons = []
        gpus = [n for n in caps.nodes.values() if n.get("gpus", 0) > 0]
        if not gpus:
            reasons.append("no GPU nodes")
        if gpus and not any("B200" in n.get("gpu_name", "") or "sm_100" in n.get("arch", "")
                            for n in gpus):
            reasons.append("sm_100a kernels need B200-class GPUs")
        return EngineSupportReport(self.name, not reasons, reasons)

    def candidate_plans(self, cfg, caps, req):
        plans = []
        for node, info in caps.nodes.items():
            n = int(info.get("gpus", 0))
            if n <= 0:
                continue
            for bp in plan_box(cfg, n, caps.measurements, batch=req.batch,
                               ctx=req.prompt_tokens + req.output_tokens, prompt=req.prompt_tokens,
                               mode=req.mode)[:4]:
                if not bp.fits:
                    continue
                mech = []
                if bp.tp > 1:
                    mech.append("fused_gemm_allreduce_nvlink")
                if cfg.is_moe and bp.ep > 1:
                    mech.append("expert_parallel")
                if bp.pp > 1:
                    mech.append("pipeline_nccl_p2p")
                if req.require_distributed and bp.tp * bp.pp * bp.dp == 1:
                    continue
                conf = "measured" if not bp.terms["unmeasured"] else "partial"
                plans.append(ExecutionPlan(
                    self.name, f"{node}: tp{bp.tp} ep{bp.ep} pp{bp.pp} dp{bp.dp}",
                    {"node": node, "tp": bp.tp, "ep": bp.ep, "pp": bp.pp, "dp": bp.dp},
                    bp.tokens_per_s, bp.ttft_ms, bp.step_ms, bp.score, mech, 0, conf, bp.terms))
        return plans


@dataclass
class ExternalEngineSlot:
    name: str
    binary: str
    note: str

    def probe(self, caps):
        ok = shutil.which(self.binary) is not None
        return EngineSupportReport(self.name, False,
                                   [self.note] + ([] if ok else [f"{self.binary} not installed"]))

    def candidate_plans(self, cfg, caps, req):
        return []


CONFIDENCE = {"measured": 1.0, "partial": 0.96, "assumed": 0.88}
WAN_FACTOR = 0.94

DEFAULT_POLICY = {
    "fused_gemm_allreduce_nvlink": Policy.AVAILABLE_CONDITIONAL,
    "expert_parallel": Policy.AVAILABLE_CONDITIONAL,
    "pipeline_nccl_p2p": Policy.AVAILABLE_CONDITIONAL,
    "speculative_decoding": Policy.EVIDENCE_ONLY,
    "lossy_activation_compression": Policy.REJECTED_DEFAULT,
}


@dataclass
class Competition:
    winner: ExecutionPlan | None
    ranked: list[ExecutionPlan]
    reports: list[EngineSupportReport]
    rejected: list[tuple[str, str]]


class EngineRegistry:
    def __init__(self, engines=None, policy=None):
        self.engines = list(engines or [
            NativeStageEngine(),
            ExternalEngineSlot("llama.cpp-rpc", "llama-server",
                               "external GGUF engine; not part of the sm_100a path"),
            ExternalEngineSlot("sglang", "sglang", "external engine; library kernels"),
        ])
        self.policy = dict(DEFAULT_POLICY, **(policy or {}))

    def compete(self, cfg: ModelConfig, caps: ClusterCapabilities, req: RequestShape) -> Competition:
        reports, ranked, rejected = [], [], []
        for e in self.engines:
            rep = e.probe(caps)
            reports.append(rep)
            if not rep.available:
                rejected.append((e.name, "; ".join(rep.reasons)))
                continue
            for p in e.candidate_plans(cfg, caps, req):
                bad = [m for m in p.mechanisms if self.policy.get(m) in (Policy.REJECTED_DEFAULT,
                                                                        Policy.EVIDENCE_ONLY)]
                if bad:
                    rejected.append((p.description, f"policy rejects {bad}"))
                    continue
                p.score *= CONFIDENCE.get(p.confidence, 0.88) * WAN_FACTOR ** p.wan_boundaries
                ranked.append(p)
        ranked.sort(key=lambda p: (-p.score, p.description))
        return Competition(ranked[0] if ranked else None, ranked, reports, rejected)
