"""Coordinator service: worker registration and heartbeats, planning, transactional
deployment onto registered workers, streamed submission with restart-and-replay, stage-0
token publication, and the gRPC server / client around them.

    CoordinatorCore         the state machine (this process's registry, deployments, requests)
    CoordinatorRpcServer    ``swarm.v1.Coordinator`` over gRPC (mutual TLS with the cluster CA)
    CoordinatorClient       what ``swarm run`` / ``swarm submit`` / workers call
    GrpcWorkerAgent         ``WorkerAgent`` (coordinator/deployment.py) over a worker's gRPC

A worker registers with its worker id, identity fingerprint and endpoints; with a cluster
state store the fingerprint must belong to a paired, unrevoked member and match the
identity bound in the caller's client certificate.  Heartbeats keep it healthy; a sweep
marks silent workers unhealthy.  ``deploy`` plans contiguous layer intervals over healthy
workers (one stage per worker, equal split or the planner's partition) and runs the
deployment manager's phases; every stage receives one lease the coordinator signs.
``submit_stream`` drives a session over the stage ring (``SessionController``); on a
transport failure it probes the route's stages, replaces the failed worker with a healthy
spare (``DeploymentManager.recover``: load, new generation, signed routes, handshakes) and
replays the request, checking every accepted token.

Reference: si/coordinator/service.py:229 (``CoordinatorCore``: :563 register, :662
heartbeat, :750 deploy, :1050 token publication, :1884 submit_stream, :1427 failed-stage
probe, :1486 recovery), :2553 (``CoordinatorRpcServer``), :3421 (``CoordinatorClient``).
"""
from __future__ import annotations

import asyncio
import json
import time
import uuid
from dataclasses import dataclass, field
from pathlib import Path

from ..protocol import stage_ring as sr
from ..telemetry.metrics import METRICS
from ..runtime.worker_runtime import COORDINATOR_SERVICE, WORKER_SERVICE, artifact_id_for
from ..transport.grpc_control import PEER_FINGERPRINT, GrpcControlClient, GrpcControlServer
from ..transport.stage_ring_net import ConnectionPool, TransportError
from .deployment import Deployment, DeploymentError, DeploymentManager, LoadReport, StagePlan
from .session import Route, SessionController
from .state import DurableState, WorkerRecord, WorkerRegistry


class GrpcWorkerAgent:
    """``WorkerAgent`` over a worker's ``swarm.v1.Worker`` gRPC service."""

    def __init__(self, worker_id: str, fingerprint: str, ring_endpoint: str, control_endpoint: str,
                 *, credentials=None, timeout: float = 60.0):
        self.worker_id = worker_id
        self.fingerprint = fingerprint
        self.endpoint = ring_endpoint           # data plane (stage ring)
        self.control_endpoint = control_endpoint
        self.client = GrpcControlClient(control_endpoint, credentials, timeout=timeout)
        self.model: dict = {}
        self.model_revision = ""
        self.num_stages = 1

    async def _call(self, method: str, kind: str, obj: dict) -> dict:
        _, rep = await self.client.call(WORKER_SERVICE, method, kind, obj)
        return rep

    async def reserve(self, deployment_id: str, stage_id: int) -> bool:
        return bool((await self._call("Reserve", "ReserveRequest",
                                      {"deployment_id": deployment_id, "stage_id": stage_id}))["ok"])

    async def release(self, deployment_id: str) -> None:
        await self._call("Release", "ReleaseRequest", {"deployment_id": deployment_id})

    async def has_artifact(self, artifact_id: str) -> bool:
        return bool((await self._call("HasArtifact", "ArtifactQuery",
                                      {"artifact_id": artifact_id}))["present"])

    async def fetch_artifact(self, artifact_id: str) -> None:
        await self._call("FetchArtifact", "ArtifactQuery", {"artifact_id": artifact_id})

    async def verify_artifact(self, artifact_id: str) -> bool:
        rep = await self._call("VerifyArtifact", "ArtifactQuery", {"artifact_id": artifact_id})
        return bool(rep.get("ok")) and bool(rep.get("present"))

    async def load_stage(self, plan: StagePlan) -> LoadReport:
        rep = await self._call("LoadStage", "LoadStageRequest", {
            "plan": {"stage_id": plan.stage_id, "layer_start": plan.layer_start,
                     "layer_end": plan.layer_end, "artifact_id": plan.artifact_id},
            "model": self.model, "model_revision": self.model_revision,
            "num_stages": self.num_stages, "deployment_id": plan.deployment_id})
        return LoadReport(rep["artifact_id"], int(rep["tensors"]), int(rep["bytes"]))

    async def unload_stage(self, deployment_id: str) -> None:
        await self._call("UnloadStage", "UnloadStageRequest", {"deployment_id": deployment_id})

    async def install_route(self, signed_lease: dict, next_endpoint: str | None) -> None:
        rep = await self._call("InstallRoute", "InstallRouteRequest",
                               {"lease": signed_lease, "next_endpoint": next_endpoint})
        if not rep.get("ok"):
            raise DeploymentError(f"{self.worker_id} rejected the route: {rep.get('error')}")

    async def withdraw_route(self, generation: int) -> None:
        await self._call("WithdrawRoute", "WithdrawRouteRequest", {"generation": generation})

    async def check_peer(self, endpoint: str) -> bool:
        rep = await self._call("CheckPeer", "CheckPeerRequest", {"endpoint": endpoint})
        if not rep.get("ok"):
            raise DeploymentError(f"{self.worker_id} handshake with {endpoint}: {rep.get('error')}")
        return True

    async def free_bytes(self) -> int:
        return int((await self._call("FreeBytes", "FreeBytesRequest", {}))["bytes"])

    async def health(self) -> dict:
        return await self._call("Health", "HealthRequest", {})

    async def close(self) -> None:
        await self.client.close()


@dataclass
class ActiveModel:
    """A deployed model: one pipeline per replica, and the scheduler that places requests
    on them (least predicted completion time among replicas with free capacity)."""
    name: str
    model: dict
    revision: str
    replicas: dict          # route id -> Deployment
    num_layers: int
    topology_id: str
    scheduler: object = None
    eos_token_ids: tuple = ()
    tokenizer: object = None       # the checkpoint's tokenizer, when it carries one

    @property
    def deployment(self) -> Deployment:
        return next(iter(self.replicas.values()))


@dataclass
class RequestRecord:
    request_id: str
    prompt: list[int]
    tokens: list[int] = field(default_factory=list)
    published: list[dict] = field(default_factory=list)
    generations: list[int] = field(default_factory=list)
    state: str = "RUNNING"
    model: str = ""
    started_at: float = 0.0
    error: str | None = None
    cancel_requested: bool = False
    replica: str | None = None
    stop_reason: str | None = None


def _model_config(model: dict):
    """The ``ModelConfig`` of a model description (a checkpoint directory or a preset)."""
    if "checkpoint" in model:
        from ..model_io.loader import checkpoint_config
        return checkpoint_config(model["checkpoint"])
    from ..models.config import preset
    return preset(model["preset"])


def model_revision(model: dict) -> str:
    return "sha256:" + __import__("hashlib").sha256(
        json.dumps(model, sort_keys=True).encode()).hexdigest()[:16]


class CoordinatorCore:
    def __init__(self, identity, *, state_dir: str | Path | None = None, cluster_store=None,
                 heartbeat_timeout_s: float = 5.0, heartbeat_s: float = 1.0,
                 worker_credentials=None, require_member: bool | None = None):
        self.identity = identity
        self.registry = WorkerRegistry(heartbeat_timeout_s)
        self.heartbeat_s = heartbeat_s
        self.agents: dict[str, GrpcWorkerAgent] = {}
        self.state = DurableState(Path(state_dir) / "coordinator_state.json") if state_dir else None
        self.deployer = DeploymentManager(self.registry, self.agents, identity, self.state)
        self.cluster_store = cluster_store
        self.require_member = cluster_store is not None if require_member is None else require_member
        self.worker_credentials = worker_credentials
        self.models: dict[str, ActiveModel] = {}
        self.requests: dict[str, RequestRecord] = {}
        self.events: list[dict] = []
        self.started_at = time.time()
        self.last_error: str | None = None
        self.pairing = None          # PairingManager when serving a cluster
        self.draining: set[str] = set()      # leaving: no new stages, never a spare
        self.unreachable: set[str] = set()   # advertised control endpoint does not answer
        self.departed: set[str] = set()      # left or removed: heartbeats refused
        self.accepting = True                # False while draining for a shutdown
        self._sweeper: asyncio.Task | None = None
        self._lock = asyncio.Lock()

    # ------------------------------------------------------------ membership
    def _check_member(self, fingerprint: str) -> None:
        if not self.require_member:
            return
        doc = self.cluster_store.load_cluster()
        members = {m["fingerprint"] for m in doc.get("members", {}).values()}
        members |= set(doc.get("trusted", {}))       # `swarm identity trust`
        revoked = set(doc.get("revoked", []))
        if fingerprint not in members or fingerprint in revoked:
            raise PermissionError("worker is neither a paired member nor trusted by this "
                                  "cluster (or is revoked)")

    def _check_caller(self, claimed: str) -> None:
        peer = PEER_FINGERPRINT.get()
        if peer is not None and peer != claimed:
            raise PermissionError("request fingerprint does not match the client certificate")
        self._check_member(claimed)

    async def register(self, req: dict) -> dict:
        self._check_caller(req["fingerprint"])
        wid = req["worker_id"]
        old = self.agents.pop(wid, None)
        if old is not None:
            await old.close()
        self.departed.discard(wid)            # an explicit registration rejoins
        self.draining.discard(wid)
        self._sync_excluded()
        self.agents[wid] = GrpcWorkerAgent(wid, req["fingerprint"], req["ring_endpoint"],
                                           req["control_endpoint"],
                                           credentials=self.worker_credentials)
        self.registry.register(WorkerRecord(wid, req["fingerprint"], req["ring_endpoint"],
                                            dict(req.get("capabilities", {}),
                                                 control_endpoint=req["control_endpoint"])))
        reachable = await self._probe(wid)
        self.events.append({"event": "worker_registered", "worker": wid, "reachable": reachable,
                            "at": time.time()})
        METRICS.inc("coordinator_registrations")
        METRICS.set("coordinator_workers_healthy", len(self.registry.healthy()))
        return {"accepted": True, "heartbeat_s": self.heartbeat_s, "reachable": reachable,
                "coordinator_fingerprint": self.identity.fingerprint}

    def _sync_excluded(self) -> None:
        self.deployer.excluded = self.draining | self.unreachable

    async def _probe(self, wid: str, timeout_s: float = 1.0) -> bool:
        """Reachability of a worker's advertised control endpoint from the coordinator: two
        Health calls (the first sets up the channel); the second's round trip becomes the
        worker's ``rtt_ms``.  An unreachable worker gets no stage and is never a spare."""
        rec, ag = self.registry.workers.get(wid), self.agents.get(wid)
        if rec is None or ag is None:
            return False
        try:
            await asyncio.wait_for(ag.health(), timeout_s)
            t0 = time.perf_counter()
            await asyncio.wait_for(ag.health(), timeout_s)
            rec.capabilities["rtt_ms"] = (time.perf_counter() - t0) * 1e3
            ok = True
        except Exception:  # noqa: BLE001 - any failure means not reachable
            rec.capabilities["rtt_ms"] = None
            ok = False
        rec.capabilities["reachable"] = ok
        (self.unreachable.discard if ok else self.unreachable.add)(wid)
        self._sync_excluded()
        return ok

    async def heartbeat(self, req: dict) -> dict:
        self._check_caller(req["fingerprint"])
        wid = req["worker_id"]
        if wid in self.departed:
            return {"ok": False, "left": True}
        if wid not in self.registry.workers:
            return {"ok": False, "reregister": True}
        self.registry.heartbeat(wid)
        if wid in self.unreachable:           # re-checked until it answers
            await self._probe(wid)
        METRICS.inc("coordinator_heartbeats")
        return {"ok": True}

    def sweep(self) -> list[str]:
        dead = self.registry.sweep()
        for wid in dead:
            self.events.append({"event": "worker_lost", "worker": wid, "at": time.time()})
            METRICS.inc("coordinator_workers_lost")
        METRICS.set("coordinator_workers_healthy", len(self.registry.healthy()))
        return dead

    async def _sweep_loop(self) -> None:
        while True:
            await asyncio.sleep(self.heartbeat_s)
            self.sweep()

    def start_background(self) -> None:
        if self._sweeper is None:
            self._sweeper = asyncio.get_running_loop().create_task(self._sweep_loop())

    def workers(self) -> list[dict]:
        out = []
        for w in self.registry.workers.values():
            out.append({"worker_id": w.worker_id, "fingerprint": w.fingerprint,
                        "ring_endpoint": w.endpoint, "healthy": w.healthy,
                        "last_heartbeat": w.last_heartbeat,
                        "control_endpoint": w.capabilities.get("control_endpoint"),
                        "reachable": w.worker_id not in self.unreachable,
                        "rtt_ms": w.capabilities.get("rtt_ms"),
                        "draining": w.worker_id in self.draining})
        return sorted(out, key=lambda d: d["worker_id"])

    # ------------------------------------------------------------ planning / deployment
    def plan(self, model: dict, stages: int | None = None, replicas: int = 1) -> list[dict]:
        """Stage plans of every replica (``replica`` key): contiguous equal layer intervals,
        one stage per free healthy worker; replicas are balanced by the workers' measured
        speed (``place_replicas``)."""
        from .replicas import place_replicas
        cfg = _model_config(model)
        healthy = sorted(self.registry.healthy(), key=lambda w: w.worker_id)
        busy = {sp.worker_id for m in self.models.values() for d in m.replicas.values()
                for sp in d.stages}
        free = [w for w in healthy if w.worker_id not in busy and w.worker_id not in self.draining
                and w.worker_id not in self.unreachable]
        replicas = max(1, int(replicas))
        n = stages or max(1, len(free) // replicas)
        n = min(n, cfg.num_layers)
        if n < 1 or len(free) < n * replicas:
            raise DeploymentError(f"{replicas} replica(s) of {n} stages need {n * replicas} free "
                                  f"healthy workers; {len(free)} available")
        speed = {w.worker_id: float(w.capabilities.get("stage_tokens_per_s", 1.0)) for w in free}
        routes = place_replicas(speed, replicas, n)
        from ..runtime.worker import equal_layer_ranges
        ranges = equal_layer_ranges(cfg.num_layers, n)
        out = []
        for r in routes:
            workers = sorted(r.workers) if len(set(speed.values())) == 1 else r.workers
            for i, (lo, hi) in enumerate(ranges):
                out.append({"replica": r.route_id, "stage_id": i, "worker_id": workers[i],
                            "layer_start": lo, "layer_end": hi,
                            "artifact_id": artifact_id_for(model, lo, hi)})
        return out

    async def deploy(self, req: dict) -> dict:
        model = req["model"]
        name = req.get("name") or model.get("preset") or Path(model.get("checkpoint", "model")).name
        async with self._lock:
            if name in self.models:
                m = self.models[name]
                return self._model_status(m)
            from .replicas import AtomicRouteAllocator, ReplicaRoute, ReplicaScheduler
            plan = self.plan(model, req.get("stages"), int(req.get("replicas") or 1))
            rev = model_revision(model)
            by_rep: dict[str, list[dict]] = {}
            for p in plan:
                by_rep.setdefault(p["replica"], []).append(p)
            topology = f"{name}:{uuid.uuid4().hex[:8]}"
            deployed = await self._deploy_replicas(model, rev, by_rep, topology)
            cap = int(req.get("capacity") or 8)
            routes = [ReplicaRoute(rid, [sp.worker_id for sp in d.stages], cap, 1.0)
                      for rid, d in deployed.items()]
            tok = None
            if "checkpoint" in model:
                from ..model_io.loader import load_tokenizer
                tok = load_tokenizer(model["checkpoint"])
            m = ActiveModel(name, model, rev, deployed, plan[-1]["layer_end"], topology,
                            ReplicaScheduler(AtomicRouteAllocator(routes)),
                            _model_config(model).eos_token_ids, tok)
            self.models[name] = m
            if self.state is not None:
                self.state.record_model(name, {"model": model, "stages": len(m.deployment.stages),
                                               "replicas": len(deployed), "capacity": cap})
            self.events.append({"event": "model_deployed", "model": name, "replicas": len(deployed),
                                "generation": m.deployment.generation, "at": time.time()})
            return self._model_status(m)

    async def restore(self, *, timeout_s: float = 120.0, poll_s: float = 0.5) -> dict:
        """After a restart: redeploys every model the durable state records (same name,
        stage count and replicas) once enough free, healthy, reachable workers have
        registered again; returns ``{name: "restored" | error}``."""
        if self.state is None:
            return {}
        interrupted = self.state.mark_restart_boundaries()   # their streams ended with us
        if interrupted:
            self.events.append({"event": "requests_interrupted", "requests": interrupted,
                                "at": time.time()})
        out = {}
        t0 = time.time()
        for name, desc in self.state.models().items():
            if name in self.models:
                out[name] = "restored"
                continue
            need = int(desc["stages"]) * int(desc.get("replicas", 1))
            while True:
                busy = {sp.worker_id for m in self.models.values() for d in m.replicas.values()
                        for sp in d.stages}
                free = [w for w in self.registry.healthy() if w.worker_id not in busy
                        and w.worker_id not in self.draining and w.worker_id not in self.unreachable]
                if len(free) >= need or time.time() - t0 > timeout_s:
                    break
                await asyncio.sleep(poll_s)
            try:
                await self.deploy({"model": desc["model"], "name": name, "stages": desc["stages"],
                                   "replicas": desc.get("replicas", 1),
                                   "capacity": desc.get("capacity")})
                out[name] = "restored"
                self.events.append({"event": "model_restored", "model": name, "at": time.time()})
            except Exception as exc:  # noqa: BLE001 - reported per model
                out[name] = f"{type(exc).__name__}: {exc}"
                self.last_error = f"restore {name}: {out[name]}"
        return out

    async def _deploy_replicas(self, model: dict, rev: str, by_rep: dict[str, list[dict]],
                               topology: str) -> dict[str, Deployment]:
        """Deploys every replica's stage plans; on a failure unloads the ones it deployed."""
        deployed: dict[str, Deployment] = {}
        try:
            for rid, ps in by_rep.items():
                for p in ps:
                    ag = self.agents[p["worker_id"]]
                    ag.model, ag.model_revision, ag.num_stages = model, rev, len(ps)
                stages = [StagePlan(p["stage_id"], p["worker_id"], p["layer_start"],
                                    p["layer_end"], p["artifact_id"]) for p in ps]
                deployed[rid] = await self.deployer.deploy(
                    stages, model_revision=rev, topology_id=f"{topology}:{rid}")
        except Exception:
            for d in deployed.values():
                await self.deployer.unload(d.deployment_id)
            raise
        return deployed

    async def scale(self, req: dict) -> dict:
        """Sets a deployed model's replica count.  Growing plans the new pipelines on free
        healthy workers (same stage count, balanced by measured speed) and adds them to the
        scheduler once they are READY; shrinking unloads idle replicas only -- with fewer idle
        replicas than asked for, nothing changes."""
        from .replicas import ReplicaRoute
        name, want = req["model"], int(req["replicas"])
        if want < 1:
            raise ValueError("a deployed model keeps at least one replica")
        async with self._lock:
            m = self.models.get(name)
            if m is None:
                return {"ok": False, "reason": f"model {name} is not deployed"}
            cur = len(m.replicas)
            alloc = m.scheduler.allocator
            if want > cur:
                n_stages = len(m.deployment.stages)
                try:
                    plan = self.plan(m.model, n_stages, want - cur)
                except DeploymentError as exc:
                    return {"ok": False, "reason": str(exc)}
                used = {int(r[len("replica"):]) for r in m.replicas if r.startswith("replica")
                        and r[len("replica"):].isdigit()}
                fresh = iter(i for i in range(10 ** 6) if i not in used)
                rename: dict[str, str] = {}
                by_rep: dict[str, list[dict]] = {}
                for p in plan:
                    rid = rename.setdefault(p["replica"], f"replica{next(fresh)}")
                    by_rep.setdefault(rid, []).append(dict(p, replica=rid))
                added = await self._deploy_replicas(m.model, m.revision, by_rep, m.topology_id)
                cap = int(req.get("capacity") or max(r.capacity for r in alloc.routes.values()))
                for rid, d in added.items():
                    m.replicas[rid] = d
                    alloc.add_route(ReplicaRoute(rid, [sp.worker_id for sp in d.stages], cap, 1.0))
                self._record_scale(m)
                self.events.append({"event": "model_scaled", "model": name, "replicas": want,
                                    "added": sorted(added), "at": time.time()})
                return {"ok": True, "replicas": len(m.replicas), "added": sorted(added)}
            if want < cur:
                idle = sorted((rid for rid in m.replicas if alloc.routes[rid].active == 0),
                              key=lambda r: (len(r), r), reverse=True)
                if len(idle) < cur - want:
                    return {"ok": False, "reason": f"only {len(idle)} idle replica(s); "
                                                   f"{cur - want} must be removed"}
                removed = idle[:cur - want]
                for rid in removed:
                    alloc.remove_route(rid)
                    await self.deployer.unload(m.replicas.pop(rid).deployment_id)
                self._record_scale(m)
                self.events.append({"event": "model_scaled", "model": name, "replicas": want,
                                    "removed": removed, "at": time.time()})
                return {"ok": True, "replicas": len(m.replicas), "removed": removed}
            return {"ok": True, "replicas": cur}

    def _record_scale(self, m: ActiveModel) -> None:
        if self.state is not None:
            desc = self.state.models().get(m.name)
            if desc is not None:
                self.state.record_model(m.name, dict(desc, replicas=len(m.replicas)))

    def _model_status(self, m: ActiveModel) -> dict:
        d = m.deployment

        def stages(dep):
            return [{"stage_id": s.stage_id, "worker_id": s.worker_id,
                     "layers": [s.layer_start, s.layer_end]} for s in dep.stages]
        return {"model": m.name, "deployment_id": d.deployment_id, "phase": d.phase.value,
                "generation": d.generation, "topology_id": d.topology_id, "revision": m.revision,
                "stages": stages(d),
                "replicas": {rid: {"deployment_id": dep.deployment_id, "phase": dep.phase.value,
                                   "generation": dep.generation, "stages": stages(dep)}
                             for rid, dep in m.replicas.items()}}

    async def unload(self, req: dict) -> dict:
        async with self._lock:
            m = self.models.pop(req["model"], None)
            if m is None:
                return {"unloaded": False}
            for d in m.replicas.values():
                await self.deployer.unload(d.deployment_id)
            if self.state is not None:
                self.state.drop_model(m.name)
            return {"unloaded": True}

    def _route(self, m: ActiveModel, d: Deployment | None = None) -> Route:
        d = d or m.deployment
        s0 = d.stages[0]
        host, port = self.agents[s0.worker_id].endpoint.rsplit(":", 1)
        return Route((host, int(port)), d.generation, d.topology_id, m.revision,
                     (s0.layer_start, s0.layer_end))

    async def _failed_workers(self, m: ActiveModel, d: Deployment) -> list[str]:
        """Workers of the route that do not answer a HEALTH frame (or are marked dead)."""
        failed = []
        pool = ConnectionPool()
        try:
            for sp in d.stages:
                rec = self.registry.workers.get(sp.worker_id)
                if rec is None or not rec.healthy:
                    failed.append(sp.worker_id)
                    continue
                host, port = self.agents[sp.worker_id].endpoint.rsplit(":", 1)
                msg = sr.StageMessage(operation=sr.Operation.HEALTH, model_revision=m.revision,
                                      tokenizer_revision="none", topology_id=m.topology_id,
                                      stage_id=sp.stage_id, layer_start=sp.layer_start,
                                      layer_end=sp.layer_end, session_id="", request_id="probe",
                                      sequence_number=0, token_position=-1,
                                      source_stage=sr.COORDINATOR, destination_stage=sp.stage_id)
                try:
                    await asyncio.wait_for(pool.send(host, int(port), msg), timeout=2.0)
                except (TransportError, OSError, asyncio.TimeoutError):
                    failed.append(sp.worker_id)
        finally:
            await pool.close()
        return failed

    async def _recover(self, m: ActiveModel, d: Deployment, route: Route, exc: Exception) -> Route:
        async with self._lock:
            if d.generation != route.generation:
                return self._route(m, d)  # another request already recovered this replica
            failed = await self._failed_workers(m, d)
            if not failed:
                raise exc
            for ag in self.agents.values():   # any healthy worker may become the replacement
                ag.model, ag.model_revision = m.model, m.revision
                ag.num_stages = len(d.stages)
            for wid in failed:
                self.registry.mark_unhealthy(wid)
                self.events.append({"event": "stage_failed", "worker": wid, "at": time.time()})
                await self.deployer.recover(d.deployment_id, wid)
            self.events.append({"event": "route_recovered", "model": m.name,
                                "generation": d.generation, "at": time.time()})
            METRICS.inc("coordinator_recoveries")
            return self._route(m, d)

    # ------------------------------------------------------------ requests
    async def submit_stream(self, req: dict):
        """Async generator of stream events for one request (``accepted``, ``token`` ...,
        ``recovered``, ``completed`` / ``failed``)."""
        name = req["model"]
        m = self.models.get(name)
        if m is None:
            yield {"event": "failed", "error": f"model {name} is not deployed"}
            return
        rid = req.get("request_id") or uuid.uuid4().hex[:12]
        if not self.accepting:
            yield {"event": "failed", "request_id": rid, "error": "the coordinator is shutting down"}
            return
        if req.get("prompt_ids") is None:
            # text prompts are tokenized here, with the checkpoint's own tokenizer
            if m.tokenizer is None or req.get("prompt") is None:
                yield {"event": "failed", "request_id": rid,
                       "error": "send prompt_ids: this model has no tokenizer" if m.tokenizer is None
                       else "a request needs prompt_ids or prompt"}
                return
            req = dict(req, prompt_ids=list(m.tokenizer.encode(req["prompt"])))
        prompt = [int(t) for t in req["prompt_ids"]]
        rec = RequestRecord(rid, prompt, model=name, started_at=time.time())
        self.requests[rid] = rec
        if self.state is not None:
            self.state.record_request(rid, prompt, {"max_tokens": req.get("max_tokens")})
        max_tokens = int(req.get("max_tokens", 16))
        stop_ids = {int(t) for t in (req.get("stop_token_ids") or ())}
        if not req.get("ignore_eos"):
            stop_ids |= set(m.eos_token_ids)
        stop_reason = "length"
        try:
            grant = m.scheduler.submit(len(prompt), max_tokens)
        except Exception as exc:  # noqa: BLE001 - every replica is at capacity
            rec.state = "REJECTED"
            rec.error = f"{type(exc).__name__}: {exc}"
            yield {"event": "failed", "request_id": rid, "error": rec.error}
            return
        d = m.replicas[grant.route_id]
        rec.replica = grant.route_id
        ctl = SessionController(self._route(m, d), recover=lambda r, e: self._recover(m, d, r, e),
                                return_logits=bool(req.get("return_logits")),
                                speculate_k=int(req.get("speculate_k") or 0))
        yield {"event": "accepted", "request_id": rid, "generation": d.generation,
               "replica": grant.route_id}
        METRICS.inc("coordinator_requests")
        t0 = time.perf_counter()
        t_last = t0
        agen = ctl.stream(prompt, max_tokens, rid)
        try:
            async for ev in agen:
                if rec.cancel_requested:
                    break
                if ev["event"] == "token":
                    now = time.perf_counter()
                    METRICS.observe("coordinator_ttft_ms" if ev["index"] == 0
                                    else "coordinator_tpot_ms", (now - t_last) * 1e3)
                    METRICS.inc("coordinator_tokens")
                    t_last = now
                    rec.tokens.append(ev["token"])
                    if self.state is not None:
                        self.state.accept_token(rid, ev["token"])
                    out = {"event": "token", "index": ev["index"], "token": ev["token"]}
                    if ev.get("logits") is not None:
                        out["logits"] = [float(v) for v in ev["logits"].reshape(-1).tolist()]
                    yield out
                    if ev["token"] in stop_ids:   # the stop token is the last one emitted
                        stop_reason = "stop_token"
                        break
                elif ev["event"] in ("started", "recovered"):
                    rec.generations.append(ev["generation"])
                    if ev["event"] == "recovered":
                        yield {"event": "recovered", "generation": ev["generation"],
                               "replayed": ev["replayed"]}
            if rec.cancel_requested:
                await agen.aclose()
                await ctl.cancel_current()  # every stage drops the session and its KV
                rec.state = "CANCELLED"
                METRICS.inc("coordinator_requests_cancelled")
                yield {"event": "cancelled", "request_id": rid, "tokens": rec.tokens}
                return
            if stop_reason == "stop_token":
                await agen.aclose()
                await ctl.cancel_current(finished=True)   # every stage closes the session
            rec.state = "COMPLETED"
            rec.stop_reason = stop_reason
            done = {"event": "completed", "request_id": rid, "tokens": rec.tokens,
                    "generations": rec.generations, "seconds": time.perf_counter() - t0,
                    "stop_reason": stop_reason, "prompt_tokens": len(prompt)}
            if m.tokenizer is not None:
                done["text"] = m.tokenizer.decode(rec.tokens)
            yield done
        except Exception as exc:  # noqa: BLE001 - reported to the caller as an event
            rec.state = "FAILED"
            rec.error = self.last_error = f"{type(exc).__name__}: {exc}"
            METRICS.inc("coordinator_requests_failed")
            if isinstance(exc, TransportError):
                METRICS.inc("coordinator_transport_errors")
            yield {"event": "failed", "request_id": rid, "error": f"{type(exc).__name__}: {exc}"}
        finally:
            m.scheduler.allocator.release(grant.lease_id)
            if self.state is not None:
                self.state.set_state(rid, rec.state)
            await ctl.pool.close()

    # ------------------------------------------------------------ membership changes
    def _stages_on(self, wid: str) -> list[tuple["ActiveModel", str, Deployment]]:
        return [(m, rid, d) for m in self.models.values() for rid, d in m.replicas.items()
                if any(sp.worker_id == wid for sp in d.stages)]

    async def _move_off(self, wid: str, *, force: bool) -> list[dict]:
        """Moves every stage ``wid`` holds onto a spare (new generation per replica).  Without
        ``force`` a replica with a running request, or a stage with no spare, refuses the
        move before anything changes."""
        hosted = self._stages_on(wid)
        for m, rid, d in hosted:
            if not force and any(r.state == "RUNNING" and r.model == m.name and r.replica == rid
                                 for r in self.requests.values()):
                raise DeploymentError(f"replica {rid} of {m.name} has running requests")
            for sp in d.stages:
                if sp.worker_id == wid and not await self.deployer.eligible_replacements(d, sp):
                    raise DeploymentError(f"no spare worker for stage {sp.stage_id} of {m.name}")
        moved = []
        for m, rid, d in hosted:
            for ag in self.agents.values():
                ag.model, ag.model_revision, ag.num_stages = m.model, m.revision, len(d.stages)
            old = d.deployment_id
            await self.deployer.recover(old, wid)
            self.events.append({"event": "stage_moved", "model": m.name, "replica": rid,
                                "from": wid, "generation": d.generation, "at": time.time()})
            moved.append({"model": m.name, "replica": rid, "generation": d.generation,
                          "stages": [[sp.stage_id, sp.worker_id] for sp in d.stages]})
            ag = self.agents.get(wid)
            if ag is not None:            # best effort: the leaving worker frees its stage
                try:
                    await asyncio.wait_for(ag.unload_stage(old), timeout=5.0)
                except Exception:  # noqa: BLE001 - it may already be gone
                    pass
        return moved

    async def _drop(self, wid: str, event: str) -> None:
        self.registry.workers.pop(wid, None)
        self.draining.discard(wid)
        self.unreachable.discard(wid)
        self._sync_excluded()
        self.departed.add(wid)
        ag = self.agents.pop(wid, None)
        if ag is not None:
            await ag.close()
        self.events.append({"event": event, "worker": wid, "at": time.time()})
        METRICS.set("coordinator_workers_healthy", len(self.registry.healthy()))

    async def leave(self, req: dict) -> dict:
        """A worker leaves gracefully (``swarm node leave``): it is drained (no new stages,
        never a spare), its stages move to spares under a new generation, it is removed from
        the registry and, with a cluster state store, from the members.  Refused, with
        nothing changed, while a replica it serves has a running request (unless ``force``)
        or when a stage has no spare."""
        self._check_caller(req["fingerprint"])
        wid = req["worker_id"]
        rec = self.registry.workers.get(wid)
        if rec is None or rec.fingerprint != req["fingerprint"]:
            return {"ok": False, "reason": f"{wid} is not registered with this identity"}
        async with self._lock:
            self.draining.add(wid)
            self._sync_excluded()
            try:
                moved = await self._move_off(wid, force=bool(req.get("force")))
            except DeploymentError as exc:
                self.draining.discard(wid)
                self._sync_excluded()
                return {"ok": False, "reason": str(exc)}
            await self._drop(wid, "worker_left")
        if self.cluster_store is not None:
            doc = self.cluster_store.load_cluster()
            gone = [k for k, v in doc.get("members", {}).items() if v["fingerprint"] == req["fingerprint"]]
            for k in gone:
                doc["members"].pop(k)
            self.cluster_store.save_cluster(doc)
        return {"ok": True, "moved": moved}

    async def remove_worker(self, req: dict) -> dict:
        """Removes a worker now (``swarm cluster revoke`` on the coordinator): its stages move
        to spares even under running requests, which resume on the new route by replay."""
        wid = req["worker_id"]
        if wid not in self.registry.workers and wid not in self.agents:
            return {"ok": False, "reason": f"unknown worker {wid}"}
        async with self._lock:
            self.draining.add(wid)
            self._sync_excluded()
            try:
                moved = await self._move_off(wid, force=True)
            except DeploymentError as exc:
                self.draining.discard(wid)
                self._sync_excluded()
                return {"ok": False, "reason": str(exc)}
            await self._drop(wid, "worker_removed")
        return {"ok": True, "moved": moved}

    async def worker_metrics(self, timeout_s: float = 2.0) -> dict:
        """Every registered worker's own view (its Health call): the stage it hosts
        (layers, generation, sessions, frames, rejections, tokens, forward time) and its
        metrics snapshot; an unanswered worker shows the error."""
        async def one(wid, ag):
            try:
                h = await asyncio.wait_for(ag.health(), timeout_s)
                return wid, {"stage": {k: v for k, v in h.items() if k != "metrics"},
                             "metrics": h.get("metrics", {})}
            except Exception as exc:  # noqa: BLE001 - reported per worker
                return wid, {"error": f"{type(exc).__name__}: {exc}"}
        pairs = await asyncio.gather(*(one(w, a) for w, a in sorted(self.agents.items())))
        return dict(pairs)

    def topology(self) -> dict:
        """Workers (health, draining, measured link class) and, per deployed model and
        replica, which worker covers which layers and whether coverage is complete: every
        layer held, by healthy workers that are not draining."""
        from ..planner.topology import LinkProfile, classify
        workers = []
        for w in sorted(self.registry.workers.values(), key=lambda w: w.worker_id):
            caps = w.capabilities
            link = None
            if caps.get("rtt_ms") is not None:
                lp = LinkProfile("coordinator", w.worker_id, float(caps["rtt_ms"]),
                                 caps.get("bandwidth_MBps"))
                link = {"rtt_ms": caps["rtt_ms"], "bandwidth_MBps": caps.get("bandwidth_MBps"),
                        "domain": str(getattr(classify(lp), "value", classify(lp)))}
            workers.append({"worker_id": w.worker_id, "healthy": w.healthy,
                            "draining": w.worker_id in self.draining,
                            "reachable": w.worker_id not in self.unreachable,
                            "ring_endpoint": w.endpoint, "link": link})
        models = {}
        for name, m in self.models.items():
            reps = {}
            for rid, d in m.replicas.items():
                spans, gaps, at = [], [], 0
                ok = True
                for sp in sorted(d.stages, key=lambda s: s.layer_start):
                    w = self.registry.workers.get(sp.worker_id)
                    live = bool(w and w.healthy and sp.worker_id not in self.draining
                                and sp.worker_id not in self.unreachable)
                    ok &= live
                    if sp.layer_start > at:
                        gaps.append([at, sp.layer_start])
                    at = max(at, sp.layer_end)
                    spans.append({"layers": [sp.layer_start, sp.layer_end],
                                  "worker_id": sp.worker_id, "live": live})
                if at < m.num_layers:
                    gaps.append([at, m.num_layers])
                reps[rid] = {"generation": d.generation, "phase": d.phase.value, "stages": spans,
                             "gaps": gaps, "complete": ok and not gaps}
            models[name] = {"layers": m.num_layers, "replicas": reps,
                            "complete": all(r["complete"] for r in reps.values())}
        return {"workers": workers, "models": models,
                "departed": sorted(self.departed), "draining": sorted(self.draining)}

    async def publish_token(self, pub: dict) -> dict:
        """Stage 0's copy of every token it relayed (checked against the accepted stream)."""
        rec = self.requests.get(pub.get("request_id", ""))
        if rec is None:
            return {"ok": False}
        rec.published.append(pub)
        return {"ok": True}

    def cancel(self, req: dict) -> dict:
        """Stops a running request before its next token; its stream ends with a
        ``cancelled`` event and every stage drops the session."""
        rec = self.requests.get(req.get("request_id", ""))
        if rec is None or rec.state != "RUNNING":
            return {"ok": False, "state": rec.state if rec else None}
        rec.cancel_requested = True
        return {"ok": True, "state": rec.state}

    def status(self) -> dict:
        """Identity, uptime, capacity, request counts, throughput and recoveries, plus one
        record per deployed model and per request (the ``status`` / ``sessions`` commands)."""
        uptime = time.time() - self.started_at
        tokens = sum(len(r.tokens) for r in self.requests.values())
        return {"coordinator_fingerprint": self.identity.fingerprint,
                "uptime_s": uptime,
                "workers": len(self.registry.workers),
                "healthy_workers": len(self.registry.healthy()),
                "active_requests": sum(r.state == "RUNNING" for r in self.requests.values()),
                "generated_tokens": tokens,
                "throughput_tokens_s": tokens / uptime if uptime > 0 else 0.0,
                "recoveries": sum(max(0, len(r.generations) - 1) for r in self.requests.values()),
                "last_error": self.last_error,
                "accepting": self.accepting,
                "draining_workers": sorted(self.draining),
                "unreachable_workers": sorted(self.unreachable),
                "departed_workers": sorted(self.departed),
                "models": {k: self._model_status(v) for k, v in self.models.items()},
                "requests": {k: {"state": r.state, "model": r.model, "prompt_tokens": len(r.prompt),
                                 "tokens": len(r.tokens), "published": len(r.published),
                                 "generations": r.generations, "started_at": r.started_at,
                                 "replica": r.replica, "stop_reason": r.stop_reason,
                                 "error": r.error}
                             for k, r in self.requests.items()}}

    async def drain(self, timeout_s: float = 30.0, poll_s: float = 0.05) -> int:
        """Stops admitting requests and waits up to ``timeout_s`` for the running ones to
        finish; returns how many were still running."""
        self.accepting = False
        t0 = time.time()
        while True:
            running = sum(r.state == "RUNNING" for r in self.requests.values())
            if running == 0 or time.time() - t0 >= timeout_s:
                break
            await asyncio.sleep(poll_s)
        self.events.append({"event": "drained", "still_running": running, "at": time.time()})
        return running

    async def close(self) -> None:
        if self._sweeper is not None:
            self._sweeper.cancel()
            try:
                await self._sweeper
            except (asyncio.CancelledError, Exception):  # noqa: BLE001
                pass
        for ag in self.agents.values():
            await ag.close()


class CoordinatorRpcServer:
    """``swarm.v1.Coordinator`` over gRPC (``Any`` envelopes with JSON bodies)."""

    def __init__(self, core: CoordinatorCore, *, host: str = "127.0.0.1", port: int = 0,
                 credentials=None):
        self.core = core

        def unary(fn, reply_kind):
            async def h(kind, obj):
                return reply_kind, await fn(obj)
            return h

        async def workers(obj):
            return {"workers": core.workers()}

        async def cancel(obj):
            return core.cancel(obj)

        async def status(obj):
            return core.status()

        async def metrics(obj):
            rep = {"snapshot": METRICS.snapshot(), "prometheus": METRICS.prometheus()}
            if obj.get("workers"):
                rep["workers"] = await core.worker_metrics()
            return rep

        async def plan(obj):
            return {"plan": core.plan(obj["model"], obj.get("stages"), int(obj.get("replicas") or 1))}

        async def pairing_create(obj):
            if core.pairing is None:
                raise PermissionError("this coordinator does not serve pairing")
            if PEER_FINGERPRINT.get() not in (None, core.identity.fingerprint):
                raise PermissionError("only the coordinator's own identity mints invitations")
            inv = core.pairing.invite(float(obj.get("ttl_s", 600.0)))
            return {"uri": inv.uri()}

        async def submit_stream(kind, obj):
            async for ev in core.submit_stream(obj):
                yield "StreamEvent", ev

        async def topology(obj):
            return core.topology()

        async def scale(obj):
            return await core.scale(obj)

        async def remove_worker(obj):
            if PEER_FINGERPRINT.get() not in (None, core.identity.fingerprint):
                raise PermissionError("only the coordinator's own identity removes workers")
            return await core.remove_worker(obj)

        handlers = {
            ("Register", "RegistrationAccepted", core.register),
            ("Heartbeat", "HeartbeatReply", core.heartbeat),
            ("DeployModel", "DeploymentStatus", core.deploy),
            ("UnloadModel", "UnloadReply", core.unload),
            ("PublishToken", "PublishReply", core.publish_token),
            ("Workers", "WorkersReply", workers),
            ("CancelRequest", "CancelReply", cancel),
            ("Status", "CoordinatorStatus", status),
            ("PlanModel", "PlanReply", plan),
            ("PairingCreate", "PairingInvitation", pairing_create),
            ("Metrics", "MetricsReply", metrics),
            ("NodeLeave", "NodeLeaveReply", core.leave),
            ("RemoveWorker", "RemoveWorkerReply", remove_worker),
            ("Topology", "TopologyStatus", topology),
            ("ScaleModel", "ScaleReply", scale),
        }
        self.server = GrpcControlServer(
            {(COORDINATOR_SERVICE, m): unary(fn, rk) for m, rk, fn in handlers},
            server_streams={(COORDINATOR_SERVICE, "SubmitStream"): submit_stream},
            host=host, port=port, credentials=credentials)

    async def start(self) -> int:
        self.core.start_background()
        return await self.server.start()

    async def stop(self) -> None:
        await self.server.stop()
        await self.core.close()


class CoordinatorClient:
    def __init__(self, target: str, credentials=None, timeout: float = 300.0):
        self.client = GrpcControlClient(target, credentials, timeout=timeout)

    async def _call(self, method: str, kind: str, obj: dict) -> dict:
        _, rep = await self.client.call(COORDINATOR_SERVICE, method, kind, obj)
        return rep

    async def deploy(self, model: dict, *, name: str | None = None, stages: int | None = None,
                     replicas: int = 1) -> dict:
        return await self._call("DeployModel", "DeployRequest",
                                {"model": model, "name": name, "stages": stages,
                                 "replicas": replicas})

    async def unload(self, name: str) -> dict:
        return await self._call("UnloadModel", "UnloadRequest", {"model": name})

    async def cancel(self, request_id: str) -> dict:
        return await self._call("CancelRequest", "CancelRequestMsg", {"request_id": request_id})

    async def workers(self) -> list[dict]:
        return (await self._call("Workers", "WorkersRequest", {}))["workers"]

    async def status(self) -> dict:
        return await self._call("Status", "StatusRequest", {})

    async def plan(self, model: dict, stages: int | None = None) -> list[dict]:
        return (await self._call("PlanModel", "PlanRequest", {"model": model, "stages": stages}))["plan"]

    async def metrics(self, *, workers: bool = False) -> dict:
        return await self._call("Metrics", "MetricsRequest", {"workers": workers})

    async def topology(self) -> dict:
        return await self._call("Topology", "TopologyRequest", {})

    async def scale(self, name: str, replicas: int) -> dict:
        return await self._call("ScaleModel", "ScaleRequest", {"model": name, "replicas": replicas})

    async def leave(self, worker_id: str, fingerprint: str, *, force: bool = False) -> dict:
        return await self._call("NodeLeave", "NodeLeaveRequest",
                                {"worker_id": worker_id, "fingerprint": fingerprint, "force": force})

    async def remove_worker(self, worker_id: str) -> dict:
        return await self._call("RemoveWorker", "RemoveWorkerRequest", {"worker_id": worker_id})

    async def pairing_uri(self, ttl_s: float = 600.0) -> str:
        return (await self._call("PairingCreate", "PairingRequest", {"ttl_s": ttl_s}))["uri"]

    async def submit_stream(self, model: str, prompt_ids: list[int] | None, max_tokens: int, *,
                            return_logits: bool = False, request_id: str | None = None,
                            speculate_k: int = 0, stop_token_ids=(), ignore_eos: bool = False,
                            prompt: str | None = None):
        """``prompt_ids``, or None with a text ``prompt`` the coordinator tokenizes with the
        deployed checkpoint's tokenizer (the ``completed`` event then carries ``text``)."""
        async for _, ev in self.client.call_stream(
                COORDINATOR_SERVICE, "SubmitStream", "SubmitRequest",
                {"model": model, "prompt_ids": None if prompt_ids is None else list(prompt_ids),
                 "prompt": prompt, "max_tokens": max_tokens,
                 "return_logits": return_logits, "request_id": request_id,
                 "speculate_k": speculate_k, "stop_token_ids": list(stop_token_ids),
                 "ignore_eos": ignore_eos}):
            yield ev

    async def close(self) -> None:
        await self.client.close()
