"""Transactional deployment of a stage plan onto workers.

Phases (each recorded in the durable audit log before it starts):

    RESERVING            reserve every assigned worker for this deployment
    PREPARING            make sure each worker holds its stage artifact ...
    TRANSFERRING         ... copying it from the source store when missing (resumable)
    VERIFYING_ARTIFACTS  artifact digests on every worker
    LOADING              stage owners load their layer intervals
    VERIFYING_LOADS      load reports (artifact id, tensor count, bytes) match the plan
    INSTALLING_ROUTES    a signed route lease with a fresh generation on every stage
    VERIFYING_PEERS      each stage reaches its next hop
    READY

Any failure rolls back what was done, in reverse (routes withdrawn, stages unloaded,
reservations released) and leaves the deployment FAILED with the error.  ``recover``
replaces a failed worker with an eligible healthy one (not in the deployment, enough
free memory), redeploys that stage and reinstalls routes on every stage under the next
generation.  ``unload`` tears a READY deployment down.

Workers are driven through the small ``WorkerAgent`` interface so the same manager
runs in-process (tests, single box) or over the control transport.

Reference: si/coordinator/deployment.py:293 ``DeploymentManager`` (:641 deploy, :1061
recover, :1421 rollback, :1000 eligible replacements, :426 signed route lease); phase
names si/protocol/product.py:420-434.
"""
from __future__ import annotations

import enum
import time
import uuid
from dataclasses import dataclass, field
from typing import Protocol

from ..security.identity import Identity, RouteLease, StageAssignment, issue_lease
from .state import DurableState, WorkerRegistry


class Phase(str, enum.Enum):
    RESERVING = "RESERVING"
    PREPARING = "PREPARING"
    TRANSFERRING = "TRANSFERRING"
    VERIFYING_ARTIFACTS = "VERIFYING_ARTIFACTS"
    LOADING = "LOADING"
    VERIFYING_LOADS = "VERIFYING_LOADS"
    INSTALLING_ROUTES = "INSTALLING_ROUTES"
    VERIFYING_PEERS = "VERIFYING_PEERS"
    READY = "READY"
    FAILED = "FAILED"
    UNLOADED = "UNLOADED"


class DeploymentError(RuntimeError):
    pass


@dataclass
class StagePlan:
    stage_id: int
    worker_id: str
    layer_start: int
    layer_end: int
    artifact_id: str
    artifact_bytes: int = 0
    deployment_id: str = ""


@dataclass
class LoadReport:
    artifact_id: str
    tensors: int
    bytes: int


class WorkerAgent(Protocol):
    """What the deployment manager needs from a worker (in-process or remote)."""

    worker_id: str
    fingerprint: str
    endpoint: str

    async def reserve(self, deployment_id: str, stage_id: int) -> bool: ...
    async def release(self, deployment_id: str) -> None: ...
    async def has_artifact(self, artifact_id: str) -> bool: ...
    async def fetch_artifact(self, artifact_id: str) -> None: ...
    async def verify_artifact(self, artifact_id: str) -> bool: ...
    async def load_stage(self, plan: StagePlan) -> LoadReport: ...
    async def unload_stage(self, deployment_id: str) -> None: ...
    async def install_route(self, signed_lease: dict, next_endpoint: str | None) -> None: ...
    async def withdraw_route(self, generation: int) -> None: ...
    async def check_peer(self, endpoint: str) -> bool: ...
    async def free_bytes(self) -> int: ...


@dataclass
class Deployment:
    deployment_id: str
    model_revision: str
    topology_id: str
    stages: list[StagePlan]
    phase: Phase = Phase.RESERVING
    generation: int = 0
    error: str = ""
    history: list[tuple[str, float]] = field(default_factory=list)
    reports: dict[int, LoadReport] = field(default_factory=dict)


class DeploymentManager:
    def __init__(self, registry: WorkerRegistry, agents: dict[str, WorkerAgent], identity: Identity,
                 state: DurableState | None = None, *, lease_ttl_s: float = 3600.0):
        self.registry = registry
        self.agents = agents
        self.identity = identity
        self.state = state
        self.ttl = lease_ttl_s
        self.deployments: dict[str, Deployment] = {}
        # Route generations fence stale routes, so they never repeat: a restarted coordinator
        # continues above the last one it handed out (kept in the durable state), and above
        # the wall clock in seconds when it has no state.
        last = int(state.data.get("last_generation", 0)) if state is not None else 0
        self._generation = max(int(time.time()), last)
        self.excluded: set[str] = set()       # draining workers: never a replacement

    # ------------------------------------------------------------ helpers
    def _enter(self, d: Deployment, phase: Phase) -> None:
        d.phase = phase
        d.history.append((phase.value, time.time()))
        if self.state is not None:
            self.state.audit("deployment_phase", deployment=d.deployment_id, phase=phase.value,
                             generation=d.generation)

    def _next_generation(self) -> int:
        self._generation += 1
        if self.state is not None:
            self.state.set_last_generation(self._generation)
        return self._generation

    def _lease(self, d: Deployment) -> dict:
        stages = []
        for sp in d.stages:
            ag = self.agents[sp.worker_id]
            stages.append(StageAssignment(sp.stage_id, sp.worker_id, ag.fingerprint, sp.layer_start,
                                          sp.layer_end, getattr(ag, "control_endpoint", ag.endpoint),
                                          ag.endpoint))
        lease = RouteLease(d.topology_id, d.generation, d.model_revision, "none", "native-stage",
                           "bf16", stages)
        return issue_lease(self.identity, lease, self.ttl)

    # ------------------------------------------------------------ deploy
    async def deploy(self, stages: list[StagePlan], *, model_revision: str, topology_id: str) -> Deployment:
        d = Deployment(uuid.uuid4().hex[:16], model_revision, topology_id,
                       sorted(stages, key=lambda s: s.stage_id))
        self.deployments[d.deployment_id] = d
        for sp in d.stages:
            sp.deployment_id = d.deployment_id
        done: list[Phase] = []
        try:
            for sp in d.stages:
                if sp.worker_id not in self.agents or not self._healthy(sp.worker_id):
                    raise DeploymentError(f"worker {sp.worker_id} unavailable")
            self._enter(d, Phase.RESERVING)
            done.append(Phase.RESERVING)  # partial reservations are released on failure too
            for sp in d.stages:
                if not await self.agents[sp.worker_id].reserve(d.deployment_id, sp.stage_id):
                    raise DeploymentError(f"worker {sp.worker_id} refused the reservation")
            await self._stage_artifacts(d, d.stages)
            self._enter(d, Phase.LOADING)
            done.append(Phase.LOADING)
            await self._load(d, d.stages)
            d.generation = self._next_generation()
            self._enter(d, Phase.INSTALLING_ROUTES)
            done.append(Phase.INSTALLING_ROUTES)
            await self._install(d)
            self._enter(d, Phase.VERIFYING_PEERS)
            await self._verify_peers(d)
            self._enter(d, Phase.READY)
            return d
        except Exception as exc:  # noqa: BLE001 - every failure rolls back
            d.error = f"{type(exc).__name__}: {exc}"
            await self._rollback(d, done)
            self._enter(d, Phase.FAILED)
            raise DeploymentError(d.error) from exc

    def _healthy(self, wid: str) -> bool:
        rec = self.registry.workers.get(wid)
        return rec is not None and rec.healthy

    async def _stage_artifacts(self, d: Deployment, stages: list[StagePlan]) -> None:
        self._enter(d, Phase.PREPARING)
        missing = [sp for sp in stages if not await self.agents[sp.worker_id].has_artifact(sp.artifact_id)]
        if missing:
            self._enter(d, Phase.TRANSFERRING)
            for sp in missing:
                await self.agents[sp.worker_id].fetch_artifact(sp.artifact_id)
        self._enter(d, Phase.VERIFYING_ARTIFACTS)
        for sp in stages:
            if not await self.agents[sp.worker_id].verify_artifact(sp.artifact_id):
                raise DeploymentError(f"artifact {sp.artifact_id} failed verification on {sp.worker_id}")

    async def _load(self, d: Deployment, stages: list[StagePlan]) -> None:
        for sp in stages:
            sp.deployment_id = d.deployment_id
            d.reports[sp.stage_id] = await self.agents[sp.worker_id].load_stage(sp)
        self._enter(d, Phase.VERIFYING_LOADS)
        for sp in stages:
            rep = d.reports[sp.stage_id]
            if rep.artifact_id != sp.artifact_id or (sp.artifact_bytes and rep.bytes != sp.artifact_bytes):
                raise DeploymentError(f"stage {sp.stage_id} loaded {rep.artifact_id} ({rep.bytes} B), "
                                      f"expected {sp.artifact_id} ({sp.artifact_bytes} B)")

    async def _install(self, d: Deployment) -> None:
        signed = self._lease(d)
        for i, sp in enumerate(d.stages):
            nxt = self.agents[d.stages[i + 1].worker_id].endpoint if i + 1 < len(d.stages) else None
            await self.agents[sp.worker_id].install_route(signed, nxt)

    async def _verify_peers(self, d: Deployment) -> None:
        for i in range(len(d.stages) - 1):
            a, b = d.stages[i], d.stages[i + 1]
            if not await self.agents[a.worker_id].check_peer(self.agents[b.worker_id].endpoint):
                raise DeploymentError(f"stage {a.stage_id} cannot reach stage {b.stage_id}")

    async def _rollback(self, d: Deployment, done: list[Phase]) -> None:
        for phase in reversed(done):
            for sp in d.stages:
                ag = self.agents.get(sp.worker_id)
                if ag is None:
                    continue
                try:
                    if phase == Phase.INSTALLING_ROUTES and d.generation:
                        await ag.withdraw_route(d.generation)
                    elif phase == Phase.LOADING:
                        await ag.unload_stage(d.deployment_id)
                    elif phase == Phase.RESERVING:
                        await ag.release(d.deployment_id)
                except Exception as exc:  # noqa: BLE001 - rollback continues past dead workers
                    if self.state is not None:
                        self.state.audit("rollback_step_failed", deployment=d.deployment_id,
                                         worker=sp.worker_id, phase=phase.value, error=str(exc))

    # ------------------------------------------------------------ recover / unload
    async def eligible_replacements(self, d: Deployment, sp: StagePlan) -> list[str]:
        used = {s.worker_id for s in d.stages}
        out = []
        for rec in self.registry.healthy():
            if rec.worker_id in used or rec.worker_id not in self.agents or rec.worker_id in self.excluded:
                continue
            if await self.agents[rec.worker_id].free_bytes() >= sp.artifact_bytes:
                out.append(rec.worker_id)
        return sorted(out)

    async def recover(self, deployment_id: str, failed_worker: str) -> Deployment:
        d = self.deployments[deployment_id]
        self.registry.mark_unhealthy(failed_worker)
        bad = [sp for sp in d.stages if sp.worker_id == failed_worker]
        if not bad:
            return d
        for sp in bad:
            cands = await self.eligible_replacements(d, sp)
            if not cands:
                d.error = f"no eligible replacement for stage {sp.stage_id}"
                self._enter(d, Phase.FAILED)
                raise DeploymentError(d.error)
            new = cands[0]
            if not await self.agents[new].reserve(d.deployment_id, sp.stage_id):
                raise DeploymentError(f"replacement {new} refused the reservation")
            sp.worker_id = new
        await self._stage_artifacts(d, bad)
        self._enter(d, Phase.LOADING)
        await self._load(d, bad)
        d.generation = self._next_generation()   # a new route generation fences the old one
        self._enter(d, Phase.INSTALLING_ROUTES)
        await self._install(d)
        self._enter(d, Phase.VERIFYING_PEERS)
        await self._verify_peers(d)
        self._enter(d, Phase.READY)
        return d

    async def unload(self, deployment_id: str) -> None:
        d = self.deployments[deployment_id]
        await self._rollback(d, [Phase.RESERVING, Phase.LOADING, Phase.INSTALLING_ROUTES])
        self._enter(d, Phase.UNLOADED)
