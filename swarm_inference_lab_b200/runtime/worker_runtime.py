"""Worker runtime of a cluster node: registration, heartbeats, a gRPC ``Worker`` control
service and a SWRING01 data-plane server that hosts the stage this node is assigned.

    swarm node agent [--state-dir DIR]         (a paired node; see ``cli.py``)

Lifecycle:

1. start the stage-ring server (data plane) and the ``swarm.v1.Worker`` gRPC service
   (control plane, mutual TLS with the cluster CA when the node holds its certificate);
2. ``Register`` with the coordinator (worker id, identity fingerprint, both endpoints,
   capabilities, free memory) and send a ``Heartbeat`` every ``heartbeat_s`` seconds;
3. serve the deployment protocol the coordinator drives (``coordinator/deployment.py``):
   Reserve / Release, HasArtifact / FetchArtifact / VerifyArtifact, LoadStage /
   UnloadStage (builds the stage owner for the assigned layer interval), InstallRoute /
   WithdrawRoute (signed leases only, verified by the stage owner), CheckPeer (the
   mutual HELLO handshake with the next stage), FreeBytes, Health;
4. stage 0 publishes every token it relays to the coordinator (``PublishToken``).

Reference: si/worker/runtime.py:113 (``WorkerRuntime``: registration, heartbeats,
control server), si/worker/stage_runtime.py:940 (route install with lease
verification), :1709-1829 (peer handshake), :2117 (bounded queue), :2468 (stage-0
token publication).
"""
from __future__ import annotations

import asyncio
import hashlib
import json
import time
from dataclasses import dataclass

import torch

from ..protocol import stage_ring as sr
from ..telemetry.metrics import METRICS
from ..transport.grpc_control import GrpcControlClient, GrpcControlServer
from ..transport.stage_ring_net import StageRingServer
from .executors import ReferenceStageExecutor, StageSpec
from .stage_owner import RouteError, RouteInfo, StageOwner

WORKER_SERVICE = "swarm.v1.Worker"
COORDINATOR_SERVICE = "swarm.v1.Coordinator"


def artifact_id_for(model: dict, layer_start: int, layer_end: int) -> str:
    """Content id of a stage: the model description plus the layer interval."""
    body = json.dumps({"model": model, "layers": [layer_start, layer_end]}, sort_keys=True)
    return hashlib.sha256(body.encode()).hexdigest()[:32]


def build_executor(model: dict, spec: StageSpec, device: str = "cpu"):
    """The stage executor for a model description: ``{"preset": name, "seed": s}`` (random
    N(0, 0.02) weights of a named architecture) or ``{"checkpoint": dir}`` (safetensors)."""
    from ..models.config import preset
    if "checkpoint" in model:
        from ..model_io.loader import checkpoint_config, safetensors_source
        cfg = checkpoint_config(model["checkpoint"])
        get = safetensors_source(model["checkpoint"])
    else:
        from ..models.reference import random_source
        cfg = preset(model["preset"])
        get = random_source(int(model.get("seed", 0)))
    backend = model.get("backend", "reference")
    if backend == "kernels":
        from .executors import KernelStageExecutor
        return cfg, KernelStageExecutor(cfg, spec, get, device=device)
    return cfg, ReferenceStageExecutor(cfg, spec, get, device=device, dtype=torch.float32)


@dataclass
class TlsFiles:
    ca: bytes
    cert: bytes
    key: bytes


class WorkerRuntime:
    def __init__(self, worker_id: str, identity, coordinator_target: str, *,
                 coordinator_fingerprint: str, host: str = "127.0.0.1", ring_port: int = 0,
                 control_port: int = 0, tls: TlsFiles | None = None, heartbeat_s: float = 1.0,
                 device: str = "cpu", free_bytes: int | None = None, max_queue: int = 64):
        self.worker_id = worker_id
        self.identity = identity
        self.coordinator_target = coordinator_target
        self.coordinator_fingerprint = coordinator_fingerprint
        self.host = host
        self.ring_port = ring_port
        self.control_port = control_port
        self.tls = tls
        self.heartbeat_s = heartbeat_s
        self.device = device
        self._free = free_bytes
        self.max_queue = max_queue
        self.owner: StageOwner | None = None
        self.ring: StageRingServer | None = None
        self.grpc: GrpcControlServer | None = None
        self.client: GrpcControlClient | None = None
        self.reservations: dict[str, int] = {}
        self.artifacts: set[str] = set()
        self.deployment_id: str | None = None
        self._hb_task: asyncio.Task | None = None
        self.heartbeats = 0
        self.registered = False

    # ------------------------------------------------------------ endpoints
    @property
    def ring_endpoint(self) -> str:
        return f"{self.host}:{self.ring_port}"

    @property
    def control_endpoint(self) -> str:
        return f"{self.host}:{self.control_port}"

    def _server_creds(self):
        if self.tls is None:
            return None
        import grpc
        return grpc.ssl_server_credentials([(self.tls.key, self.tls.cert)],
                                           root_certificates=self.tls.ca, require_client_auth=True)

    def _channel_creds(self):
        if self.tls is None:
            return None
        import grpc
        return grpc.ssl_channel_credentials(root_certificates=self.tls.ca, private_key=self.tls.key,
                                            certificate_chain=self.tls.cert)

    # ------------------------------------------------------------ lifecycle
    async def start(self) -> None:
        self.ring = StageRingServer(self._frame, host=self.host, port=self.ring_port)
        self.ring_port = await self.ring.start()
        methods = {"Reserve": self._reserve, "Release": self._release,
                   "HasArtifact": self._has_artifact, "FetchArtifact": self._fetch_artifact,
                   "VerifyArtifact": self._verify_artifact, "LoadStage": self._load_stage,
                   "UnloadStage": self._unload_stage, "InstallRoute": self._install_route,
                   "WithdrawRoute": self._withdraw_route, "CheckPeer": self._check_peer,
                   "FreeBytes": self._free_bytes, "Health": self._health}
        self.grpc = GrpcControlServer({(WORKER_SERVICE, k): v for k, v in methods.items()},
                                      host=self.host, port=self.control_port,
                                      credentials=self._server_creds())
        self.control_port = await self.grpc.start()
        self.client = GrpcControlClient(self.coordinator_target, self._channel_creds(), timeout=30.0)
        await self.register()
        self._hb_task = asyncio.get_running_loop().create_task(self._heartbeat_loop())

    async def register(self) -> dict:
        caps = {"device": self.device, "free_bytes": await self._free_bytes_value(),
                "cpu_threads": torch.get_num_threads()}
        _, rep = await self.client.call(COORDINATOR_SERVICE, "Register", "WorkerRegistration", {
            "worker_id": self.worker_id, "fingerprint": self.identity.fingerprint,
            "ring_endpoint": self.ring_endpoint, "control_endpoint": self.control_endpoint,
            "capabilities": caps}, expect="RegistrationAccepted")
        self.registered = bool(rep.get("accepted"))
        if not self.registered:
            raise RuntimeError(f"coordinator refused registration: {rep.get('reason')}")
        self.heartbeat_s = float(rep.get("heartbeat_s", self.heartbeat_s))
        return rep

    async def _heartbeat_loop(self) -> None:
        while True:
            await asyncio.sleep(self.heartbeat_s)
            try:
                _, rep = await self.client.call(COORDINATOR_SERVICE, "Heartbeat", "WorkerHeartbeat", {
                    "worker_id": self.worker_id, "fingerprint": self.identity.fingerprint,
                    "generation": self.owner.route.generation if self.owner else 0,
                    "deployment_id": self.deployment_id, "at": time.time()})
                self.heartbeats += 1
                METRICS.inc("worker_heartbeats")
                if rep.get("left"):           # this worker left or was removed
                    self.registered = False
                    return
                if rep.get("reregister"):
                    # the coordinator restarted (or forgot this worker): reservations made
                    # for its earlier deployments are void
                    self.reservations.clear()
                    await self.register()
            except asyncio.CancelledError:
                raise
            except Exception:  # noqa: BLE001 - the coordinator may be restarting
                METRICS.inc("worker_heartbeat_failures")

    async def leave(self, *, force: bool = False) -> dict:
        """Leaves the cluster gracefully: the coordinator moves this worker's stages to spares
        and forgets it; heartbeats stop.  Refused (nothing changes) while a replica it serves
        has a running request, unless ``force``."""
        _, rep = await self.client.call(COORDINATOR_SERVICE, "NodeLeave", "NodeLeaveRequest", {
            "worker_id": self.worker_id, "fingerprint": self.identity.fingerprint,
            "force": force})
        if rep.get("ok"):
            self.registered = False
            if self._hb_task is not None:
                self._hb_task.cancel()
        return rep

    async def stop(self) -> None:
        if self._hb_task is not None:
            self._hb_task.cancel()
            try:
                await self._hb_task
            except (asyncio.CancelledError, Exception):  # noqa: BLE001
                pass
        if self.owner is not None:
            await self.owner.pool.close()
        if self.grpc is not None:
            await self.grpc.stop()
        if self.ring is not None:
            await self.ring.close()
        if self.client is not None:
            await self.client.close()

    # ------------------------------------------------------------ data plane
    async def _frame(self, msg: sr.StageMessage):
        if self.owner is None:
            return [sr.StageMessage(
                operation=sr.Operation.ERROR, model_revision=msg.model_revision,
                tokenizer_revision=msg.tokenizer_revision, topology_id=msg.topology_id,
                stage_id=msg.destination_stage, layer_start=msg.layer_start,
                layer_end=msg.layer_end, session_id=msg.session_id, request_id=msg.request_id,
                sequence_number=msg.sequence_number, token_position=msg.token_position,
                source_stage=msg.destination_stage, destination_stage=msg.source_stage,
                status="ERROR", attributes={"error": "SessionError", "detail": "no stage loaded"})]
        return await self.owner.handle(msg)

    async def _publish(self, pub: dict) -> None:
        await self.client.call(COORDINATOR_SERVICE, "PublishToken", "TokenPublication",
                               dict(pub, worker_id=self.worker_id))

    # ------------------------------------------------------------ control plane
    async def _reserve(self, kind, obj):
        dep = obj["deployment_id"]
        busy = [d for d in self.reservations if d != dep]
        if busy:
            return "ReserveReply", {"ok": False, "reason": f"reserved by {busy[0]}"}
        self.reservations[dep] = int(obj["stage_id"])
        return "ReserveReply", {"ok": True}

    async def _release(self, kind, obj):
        self.reservations.pop(obj["deployment_id"], None)
        return "Ack", {}

    async def _has_artifact(self, kind, obj):
        return "ArtifactReply", {"present": obj["artifact_id"] in self.artifacts}

    async def _fetch_artifact(self, kind, obj):
        # Random-weight presets and local checkpoints need no transfer: the description is
        # the artifact.  (Checkpoint shards are read from the path named in the description.)
        self.artifacts.add(obj["artifact_id"])
        return "Ack", {}

    async def _verify_artifact(self, kind, obj):
        return "ArtifactReply", {"present": obj["artifact_id"] in self.artifacts, "ok": True}

    async def _load_stage(self, kind, obj):
        plan, model = obj["plan"], obj["model"]
        spec = StageSpec(int(plan["stage_id"]), int(plan["layer_start"]), int(plan["layer_end"]),
                         int(obj["num_stages"]))
        want = artifact_id_for(model, spec.layer_start, spec.layer_end)
        if plan["artifact_id"] != want:
            raise RuntimeError(f"artifact id {plan['artifact_id']} does not describe the stage")
        cfg, ex = await asyncio.to_thread(build_executor, model, spec, self.device)
        if self.owner is not None:
            await self.owner.pool.close()
        route = RouteInfo(topology_id="pending", generation=0,
                          model_revision=obj["model_revision"])
        self.owner = StageOwner(ex, route, identity=self.identity,
                                coordinator_fingerprint=self.coordinator_fingerprint,
                                publisher=self._publish if spec.is_first else None,
                                max_queue=self.max_queue)
        self.deployment_id = obj["deployment_id"]
        self.artifacts.add(want)
        nbytes = ex.nbytes() if hasattr(ex, "nbytes") else 0
        tensors = ex.num_tensors() if hasattr(ex, "num_tensors") else 0
        return "LoadReport", {"artifact_id": want, "tensors": tensors, "bytes": nbytes}

    async def _unload_stage(self, kind, obj):
        if self.owner is not None and self.deployment_id == obj["deployment_id"]:
            await self.owner.pool.close()
            self.owner = None
            self.deployment_id = None
        return "Ack", {}

    async def _install_route(self, kind, obj):
        if self.owner is None:
            raise RuntimeError("no stage loaded")
        try:
            gen = self.owner.install_route(obj["lease"], obj.get("next_endpoint"))
        except RouteError as exc:
            return "RouteReply", {"ok": False, "error": str(exc)}
        await self.owner.pool.close()
        return "RouteReply", {"ok": True, "generation": gen}

    async def _withdraw_route(self, kind, obj):
        if self.owner is not None:
            self.owner.withdraw_route(int(obj["generation"]))
        return "Ack", {}

    async def _check_peer(self, kind, obj):
        if self.owner is None:
            return "PeerReply", {"ok": False, "error": "no stage loaded"}
        try:
            ok = await self.owner.handshake_next()
        except Exception as exc:  # noqa: BLE001 - reported to the coordinator
            return "PeerReply", {"ok": False, "error": f"{type(exc).__name__}: {exc}"}
        return "PeerReply", {"ok": bool(ok)}

    async def _free_bytes_value(self) -> int:
        if self._free is not None:
            return self._free
        if self.device.startswith("cuda") and torch.cuda.is_available():
            return int(torch.cuda.mem_get_info()[0])
        import psutil
        return int(psutil.virtual_memory().available)

    async def _free_bytes(self, kind, obj):
        return "FreeBytesReply", {"bytes": await self._free_bytes_value()}

    async def _health(self, kind, obj):
        h = {"worker_id": self.worker_id, "heartbeats": self.heartbeats,
             "deployment_id": self.deployment_id}
        if self.owner is not None:
            h.update(self.owner.health())
        h["metrics"] = METRICS.snapshot()
        return "WorkerHealth", h
