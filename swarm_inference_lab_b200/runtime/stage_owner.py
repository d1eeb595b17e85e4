"""Persistent stage owner: loads its layer interval once and serves many sessions.

Message flow per generated token (the ring):

    coordinator --PREFILL/DECODE--> stage 0 --> stage 1 --> ... --> last stage
    coordinator <--TOKEN_RESULT---- stage 0 <-- stage 1 <-- ... <-- (greedy token)

Each stage validates the frame (model revision, topology, route generation,
session, strict per-edge sequence numbers), runs its executor, and either
forwards the boundary activation to the next stage and relays the
TOKEN_RESULT back, or (last stage) selects the token and answers.  Sessions
are opened on every stage by forwarding OPEN_SESSION down the ring, so the
coordinator talks to stage 0 only and never relays hidden states.

Reference: si/worker/stage_runtime.py:213 (``PersistentStageRuntime``):
:1391 open_session, :1960 handle_message, :2137 _execute_message,
:2221 forward, :2276 token result, :2428 relay.
"""
from __future__ import annotations

import asyncio
import time
from dataclasses import dataclass, field

import torch

from ..protocol import stage_ring as sr
from ..telemetry.metrics import METRICS
from ..transport.stage_ring_net import ConnectionPool, TransportError
from ..transport.tensor_codec import pack_tensor, unpack_tensor
from .executors import StageExecutor


@dataclass
class RouteInfo:
    topology_id: str
    generation: int
    model_revision: str
    tokenizer_revision: str = "none"
    next_hop: tuple[str, int] | None = None
    next_stage: int | None = None
    # From the installed signed lease: who may talk to this stage and who it talks to.
    prev_fingerprint: str | None = None
    next_fingerprint: str | None = None


# Rows of one VERIFY_CANDIDATES frame (the last accepted token plus the draft).
MAX_VERIFY_ROWS = 64


class BackpressureError(RuntimeError):
    """The stage's bounded execution queue is full; the caller should retry later."""


class RouteError(RuntimeError):
    """A route lease or peer handshake was rejected."""


def hello_record(identity, *, topology_id: str, generation: int, stage_id: int, to_stage: int,
                 nonce: str) -> dict:
    """A signed HELLO body: proves the sender holds the identity the lease names for its
    stage, for this topology and generation, towards one receiving stage."""
    from ..security.identity import sign_record
    return sign_record(identity, {"kind": "stage_hello", "topology_id": topology_id,
                                  "generation": generation, "stage_id": stage_id,
                                  "to_stage": to_stage, "nonce": nonce, "at": time.time()})


def check_hello(rec: dict, *, expect_fingerprint: str, topology_id: str, generation: int,
                stage_id: int, to_stage: int, nonce: str | None = None,
                max_skew_s: float = 300.0) -> None:
    from ..security.identity import SignatureError, verify_record
    try:
        body = verify_record(rec, {expect_fingerprint})
    except SignatureError as exc:
        raise RouteError(f"hello: {exc}") from None
    if body.get("kind") != "stage_hello" or body.get("topology_id") != topology_id:
        raise RouteError("hello: wrong kind or topology")
    if body.get("generation") != generation:
        raise RouteError(f"hello: generation {body.get('generation')} != installed {generation}")
    if body.get("stage_id") != stage_id or body.get("to_stage") != to_stage:
        raise RouteError("hello: wrong stage pair")
    if nonce is not None and body.get("nonce") != nonce:
        raise RouteError("hello: nonce mismatch")
    if abs(time.time() - float(body.get("at", 0))) > max_skew_s:
        raise RouteError("hello: stale timestamp")


@dataclass
class OwnerStats:
    sessions_opened: int = 0
    sessions_closed: int = 0
    frames: int = 0
    rejected: int = 0
    forward_ms: float = 0.0
    tokens: int = 0
    relayed: int = 0
    errors: list = field(default_factory=list)


class StageOwner:
    def __init__(self, executor: StageExecutor, route: RouteInfo, *, max_queue: int = 64,
                 compression: str = "none", pool: ConnectionPool | None = None,
                 identity=None, coordinator_fingerprint: str | None = None, publisher=None):
        self.ex = executor
        self.spec = executor.spec
        self.route = route
        self.pool = pool or ConnectionPool()
        # Signed-route mode: with an identity and the coordinator's fingerprint, routes are
        # installed only from leases the coordinator signed, and a stage's predecessor must
        # complete a HELLO handshake before frames of the installed generation are served.
        self.identity = identity
        self.coordinator_fingerprint = coordinator_fingerprint
        self.verifier = None
        if coordinator_fingerprint is not None:
            from ..security.identity import LeaseVerifier
            self.verifier = LeaseVerifier(coordinator_fingerprint)
        self.lease = None
        self.hello_ok_generation = -1   # generation whose predecessor handshake succeeded
        self.publisher = publisher      # stage 0: async fn(dict) publishing each token
        self.max_queue = max_queue
        self._inflight = 0
        self.seq_in = sr.SequenceValidator()
        self.seq_out = sr.SequenceAllocator()
        self.sessions = sr.SessionValidator(sr.SessionPin(
            model_revision=route.model_revision, topology_id=route.topology_id,
            stage_id=self.spec.stage_id, layer_range=(self.spec.layer_start, self.spec.layer_end)))
        self.stats = OwnerStats()
        self.compression = compression
        self._sem = asyncio.Semaphore(max_queue)
        self._lock = asyncio.Lock()  # executor calls are serialised per owner

    # ------------------------------------------------------------ helpers
    def _reply(self, req: sr.StageMessage, op: sr.Operation, *, status="OK", payload=b"",
               attrs=None, shape=(), dtype="none") -> sr.StageMessage:
        return sr.StageMessage(
            operation=op, model_revision=req.model_revision, tokenizer_revision=req.tokenizer_revision,
            topology_id=req.topology_id, stage_id=self.spec.stage_id,
            layer_start=self.spec.layer_start, layer_end=self.spec.layer_end,
            session_id=req.session_id, request_id=req.request_id,
            sequence_number=req.sequence_number, token_position=req.token_position,
            source_stage=self.spec.stage_id, destination_stage=req.source_stage,
            tensor_shape=tuple(shape), tensor_dtype=dtype, payload=payload, status=status,
            attributes=attrs or {})

    def _error(self, req: sr.StageMessage, exc: Exception) -> list[sr.StageMessage]:
        self.stats.rejected += 1
        METRICS.inc("stage_rejected_frames", stage=self.spec.stage_id, error=type(exc).__name__)
        self.stats.errors.append(f"{type(exc).__name__}: {exc}")
        return [self._reply(req, sr.Operation.ERROR, status="ERROR",
                            attrs={"error": type(exc).__name__, "detail": str(exc)})]

    def _downstream(self, req: sr.StageMessage, op: sr.Operation, *, payload=b"", attrs=None,
                    shape=(), dtype="none") -> sr.StageMessage:
        nxt = self.route.next_stage
        return sr.StageMessage(
            operation=op, model_revision=req.model_revision, tokenizer_revision=req.tokenizer_revision,
            topology_id=req.topology_id, stage_id=nxt, layer_start=self._next_range[0],
            layer_end=self._next_range[1], session_id=req.session_id, request_id=req.request_id,
            sequence_number=self.seq_out.next(req.session_id, self.spec.stage_id, nxt),
            token_position=req.token_position, source_stage=self.spec.stage_id,
            destination_stage=nxt, tensor_shape=tuple(shape), tensor_dtype=dtype,
            compression_mode=attrs.get("codec", "none") if attrs else "none", payload=payload,
            attributes=dict(attrs or {}, generation=self.route.generation))

    _next_range: tuple[int, int] = (0, 0)

    def set_next_range(self, start: int, end: int) -> None:
        self._next_range = (start, end)

    async def _send_next(self, msg: sr.StageMessage) -> sr.StageMessage:
        host, port = self.route.next_hop
        return await self.pool.send(host, port, msg)

    # ------------------------------------------------------------ dispatch
    async def handle(self, msg: sr.StageMessage) -> list[sr.StageMessage]:
        self.stats.frames += 1
        op = msg.operation
        try:
            if op == sr.Operation.HEALTH:
                return [self._reply(msg, sr.Operation.HEALTH, attrs=self.health())]
            if op == sr.Operation.HELLO:
                return [self._reply(msg, sr.Operation.HELLO, attrs=self._hello_reply(msg))]
            gen = msg.attributes.get("generation", self.route.generation)
            if gen != self.route.generation:
                raise sr.SessionError(f"stale route generation {gen} (installed "
                                      f"{self.route.generation})")
            self.sessions.check(msg)
            if (self.verifier is not None and self.spec.stage_id > 0
                    and self.hello_ok_generation != self.route.generation):
                raise sr.SessionError("no completed peer handshake for the installed route")
            if op in (sr.Operation.PREFILL, sr.Operation.DECODE, sr.Operation.VERIFY_CANDIDATES,
                      sr.Operation.CLOSE_SESSION, sr.Operation.CANCEL_SESSION):
                self.seq_in.check(msg)
        except (sr.SessionError, sr.SequenceError) as exc:
            return self._error(msg, exc)
        METRICS.inc("stage_frames", stage=self.spec.stage_id, op=op.name)
        if self._inflight >= self.max_queue:
            self.stats.rejected += 1
            METRICS.inc("stage_backpressure", stage=self.spec.stage_id)
            return [self._reply(msg, sr.Operation.ERROR, status="ERROR", attrs={
                "error": "BackpressureError", "detail": f"execution queue full ({self.max_queue})",
                "retry_after_ms": 5})]
        self._inflight += 1
        try:
            return await self._dispatch(msg)
        finally:
            self._inflight -= 1

    async def _dispatch(self, msg: sr.StageMessage) -> list[sr.StageMessage]:
        op = msg.operation
        async with self._sem:
            try:
                if op == sr.Operation.OPEN_SESSION:
                    return await self._open(msg)
                if op in (sr.Operation.CLOSE_SESSION, sr.Operation.CANCEL_SESSION):
                    return await self._close(msg)
                if op in (sr.Operation.PREFILL, sr.Operation.DECODE, sr.Operation.VERIFY_CANDIDATES):
                    return await self._execute(msg)
                raise sr.FrameError(f"unexpected operation {op.name}")
            except TransportError:
                raise
            except Exception as exc:  # noqa: BLE001 - reported back as an ERROR frame
                return self._error(msg, exc)

    async def _open(self, msg):
        async with self._lock:
            self.ex.open(msg.session_id)
        self.stats.sessions_opened += 1
        if not self.spec.is_last:
            rep = await self._send_next(self._downstream(msg, sr.Operation.OPEN_SESSION))
            if rep.status != "OK":
                return [self._reply(msg, sr.Operation.ERROR, status="ERROR", attrs=rep.attributes)]
        return [self._reply(msg, sr.Operation.OPEN_SESSION)]

    async def _close(self, msg):
        async with self._lock:
            self.ex.close(msg.session_id)
        self.seq_in.reset_session(msg.session_id)
        self.stats.sessions_closed += 1
        if not self.spec.is_last:
            # The relayed close takes the session's next outgoing sequence number (the next
            # stage rejects a restarted one as stale and would keep its session open); the
            # counter restarts only after it.
            down = self._downstream(msg, msg.operation)
            self.seq_out.reset_session(msg.session_id)
            try:
                await self._send_next(down)
            except TransportError:
                pass  # the downstream session dies with its connection
        else:
            self.seq_out.reset_session(msg.session_id)
        return [self._reply(msg, msg.operation)]

    async def _execute(self, msg):
        """PREFILL / DECODE / VERIFY_CANDIDATES: run this stage's layers on the frame's rows at
        its position and forward the activations (the last stage answers with the greedy
        token; for VERIFY_CANDIDATES with the greedy token after every row, ``tokens``).  A
        ``truncate_to`` attribute first rolls the session's cache back to that length (the
        candidates of an earlier verification that the client rejected); it travels down the
        ring with the frame."""
        attrs = msg.attributes
        x = unpack_tensor(msg.payload, attrs["tensor"])
        if msg.operation == sr.Operation.VERIFY_CANDIDATES and x.shape[0] > MAX_VERIFY_ROWS:
            raise sr.FrameError(f"{x.shape[0]} candidate rows (at most {MAX_VERIFY_ROWS})")
        t0 = time.perf_counter()
        async with self._lock:
            if attrs.get("truncate_to") is not None:
                keep = int(attrs["truncate_to"])
                have = self.ex.length(msg.session_id)
                if not 0 <= keep <= have:
                    raise sr.FrameError(f"truncate_to {keep} outside the session's {have} tokens")
                self.ex.truncate(msg.session_id, keep)
            y = await asyncio.to_thread(self.ex.forward, msg.session_id, x, msg.token_position)
        dt_ms = (time.perf_counter() - t0) * 1e3
        self.stats.forward_ms += dt_ms
        METRICS.observe("stage_forward_ms", dt_ms, stage=self.spec.stage_id)
        if self.spec.is_last:
            last = y[-1].float()
            token = int(torch.argmax(last))  # lowest id on ties
            self.stats.tokens += 1
            out_attrs = {"token": token, "replay": bool(attrs.get("replay", False))}
            if msg.operation == sr.Operation.VERIFY_CANDIDATES:
                preds = [int(t) for t in torch.argmax(y.float(), dim=-1).tolist()]
                out_attrs["tokens"] = preds
                out_attrs["token"] = preds[0]
            payload, shape, dtype = b"", (), "none"
            if attrs.get("return_logits"):
                pk = pack_tensor(last.cpu())
                out_attrs["tensor"] = pk.attributes
                payload, shape, dtype = pk.payload, pk.shape, "float32"
            return [self._reply(msg, sr.Operation.TOKEN_RESULT, attrs=out_attrs, payload=payload,
                                shape=shape, dtype=dtype)]
        pk = pack_tensor(y, compression=self.compression)
        fwd_attrs = {"tensor": pk.attributes, "codec": pk.attributes["codec"]}
        for k in ("return_logits", "replay", "truncate_to"):
            if k in attrs:
                fwd_attrs[k] = attrs[k]
        rep = await self._send_next(self._downstream(msg, msg.operation, payload=pk.payload,
                                                     attrs=fwd_attrs, shape=pk.shape,
                                                     dtype=pk.attributes["dtype"]))
        self.stats.relayed += 1
        if rep.operation == sr.Operation.ERROR:
            return [self._reply(msg, sr.Operation.ERROR, status="ERROR", attrs=rep.attributes)]
        if self.spec.is_first and self.publisher is not None and "token" in rep.attributes:
            # Stage-0 token publication: the coordinator hears every token from stage 0 too
            # (recorded next to the request; a replayed token is marked as such).
            pub = {"request_id": msg.request_id, "session_id": msg.session_id,
                   "position": msg.token_position, "token": int(rep.attributes["token"]),
                   "generation": self.route.generation,
                   "replay": bool(rep.attributes.get("replay", False))}
            asyncio.get_running_loop().create_task(self._publish(pub))
        return [self._reply(msg, sr.Operation.TOKEN_RESULT, attrs=rep.attributes,
                            payload=rep.payload, shape=rep.tensor_shape, dtype=rep.tensor_dtype)]

    async def _publish(self, pub: dict) -> None:
        try:
            await self.publisher(pub)
        except Exception as exc:  # noqa: BLE001 - publication is best effort
            self.stats.errors.append(f"publish: {type(exc).__name__}: {exc}")

    # ------------------------------------------------------------ signed routes
    def install_route(self, signed_lease: dict, next_endpoint: str | None) -> int:
        """Installs the route of a lease the coordinator signed.  Rejects unsigned, foreign,
        expired, replayed or stale-generation leases and leases that do not assign this
        worker this stage.  Returns the installed generation."""
        from ..security.identity import SignatureError
        if self.verifier is None or self.identity is None:
            raise RouteError("this stage owner has no coordinator identity to verify leases")
        try:
            lease = self.verifier.verify(signed_lease, worker_fingerprint=self.identity.fingerprint,
                                         model_revision=self.route.model_revision)
        except SignatureError as exc:
            raise RouteError(str(exc)) from None
        mine = [a for a in lease.stages if a.worker_fingerprint == self.identity.fingerprint
                and a.stage_id == self.spec.stage_id]
        if not mine:
            raise RouteError(f"lease does not assign stage {self.spec.stage_id} to this worker")
        a = mine[0]
        if (a.layer_start, a.layer_end) != (self.spec.layer_start, self.spec.layer_end):
            raise RouteError("lease layer interval differs from the loaded stage")
        by_stage = {s.stage_id: s for s in lease.stages}
        nxt = by_stage.get(self.spec.stage_id + 1)
        prev = by_stage.get(self.spec.stage_id - 1)
        if nxt is not None:
            ep = next_endpoint or nxt.data_endpoint
            if ep != nxt.data_endpoint:
                raise RouteError("next hop differs from the lease")
            host, port = ep.rsplit(":", 1)
            self.route.next_hop = (host, int(port))
            self.route.next_stage = nxt.stage_id
            self.route.next_fingerprint = nxt.worker_fingerprint
            self.set_next_range(nxt.layer_start, nxt.layer_end)
        else:
            self.route.next_hop = None
            self.route.next_stage = None
            self.route.next_fingerprint = None
        self.route.prev_fingerprint = prev.worker_fingerprint if prev else None
        self.route.topology_id = lease.topology_id
        self.route.generation = lease.generation
        self.sessions.pin.topology_id = lease.topology_id
        self.lease = lease
        return lease.generation

    def withdraw_route(self, generation: int) -> None:
        if self.route.generation == generation:
            self.route.next_hop = None
            self.hello_ok_generation = -1

    def _hello_reply(self, msg: sr.StageMessage) -> dict:
        base = {"stage_id": self.spec.stage_id, "generation": self.route.generation}
        rec = msg.attributes.get("hello")
        if self.verifier is None or rec is None:
            return base
        if self.route.prev_fingerprint is None:
            raise sr.SessionError("stage 0 accepts no peer handshake")
        check_hello(rec, expect_fingerprint=self.route.prev_fingerprint,
                    topology_id=self.route.topology_id, generation=self.route.generation,
                    stage_id=self.spec.stage_id - 1, to_stage=self.spec.stage_id)
        self.hello_ok_generation = self.route.generation
        base["hello"] = hello_record(self.identity, topology_id=self.route.topology_id,
                                     generation=self.route.generation, stage_id=self.spec.stage_id,
                                     to_stage=self.spec.stage_id - 1, nonce=rec["nonce"])
        return base

    async def handshake_next(self) -> bool:
        """HELLO to the next stage: both sides prove the identities the lease names."""
        import secrets
        if self.route.next_hop is None:
            return True
        nonce = secrets.token_hex(16)
        rec = hello_record(self.identity, topology_id=self.route.topology_id,
                           generation=self.route.generation, stage_id=self.spec.stage_id,
                           to_stage=self.route.next_stage, nonce=nonce)
        msg = sr.StageMessage(
            operation=sr.Operation.HELLO, model_revision=self.route.model_revision,
            tokenizer_revision=self.route.tokenizer_revision, topology_id=self.route.topology_id,
            stage_id=self.route.next_stage, layer_start=self._next_range[0],
            layer_end=self._next_range[1], session_id="hello", request_id="hello",
            sequence_number=0, token_position=-1, source_stage=self.spec.stage_id,
            destination_stage=self.route.next_stage, attributes={"hello": rec})
        rep = await self._send_next(msg)
        if rep.operation == sr.Operation.ERROR:
            raise RouteError(f"next stage refused the handshake: {rep.attributes.get('detail')}")
        check_hello(rep.attributes.get("hello") or {}, expect_fingerprint=self.route.next_fingerprint,
                    topology_id=self.route.topology_id, generation=self.route.generation,
                    stage_id=self.route.next_stage, to_stage=self.spec.stage_id, nonce=nonce)
        return True

    def health(self) -> dict:
        s = self.stats
        return {"stage_id": self.spec.stage_id, "layers": [self.spec.layer_start, self.spec.layer_end],
                "generation": self.route.generation, "sessions_active": len(self.sessions.active),
                "sessions_opened": s.sessions_opened, "frames": s.frames, "rejected": s.rejected,
                "tokens": s.tokens, "forward_ms": round(s.forward_ms, 3)}
