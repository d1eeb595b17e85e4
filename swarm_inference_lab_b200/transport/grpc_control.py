"""gRPC control transport: ``swarm.v1.Coordinator`` / ``swarm.v1.Worker`` services.

Control messages travel as ``google.protobuf.Any`` envelopes whose ``type_url``
is ``type.swarm-inference.dev/<Kind>`` and whose value is compact, key-sorted
JSON -- the envelope convention of the reference, so peers interoperate at the
message level.  Activation tensors stream as ``swarm.v1.Chunk`` messages
(tensor id, chunk index / count, total length, payload, SHA-256 of the whole
tensor) over a bidirectional ``ExecuteStream``; the receiver reassembles and
verifies the tensor before the handler sees it.

No generated stubs are needed: the services use gRPC generic handlers, and the
``Chunk`` message class is built from a descriptor at import time.

Reference: si/transport/grpc_transport.py:152,574; proto/swarm.proto; envelope
si/protocol/messages.py:395-420.
"""
from __future__ import annotations

import contextvars
import hashlib
import json

import grpc
from google.protobuf import any_pb2, descriptor_pb2, descriptor_pool, message_factory

TYPE_PREFIX = "type.swarm-inference.dev/"
CHUNK_BYTES = 1 << 20

# Identity fingerprint bound into the caller's client certificate (mutual TLS), set while
# a handler runs; None on an insecure server or for a certificate without the binding.
PEER_FINGERPRINT: contextvars.ContextVar[str | None] = contextvars.ContextVar(
    "peer_fingerprint", default=None)


def _peer_fingerprint(ctx) -> str | None:
    try:
        auth = ctx.auth_context()
    except Exception:  # noqa: BLE001
        return None
    pems = auth.get("x509_pem_cert") or []
    if not pems:
        return None
    from ..security.tls import cert_fingerprint_binding
    return cert_fingerprint_binding(pems[0])


class EnvelopeError(ValueError):
    pass


def pack(kind: str, obj: dict) -> any_pb2.Any:
    a = any_pb2.Any()
    a.type_url = TYPE_PREFIX + kind
    a.value = json.dumps(obj, sort_keys=True, separators=(",", ":")).encode()
    return a


def unpack(a: any_pb2.Any, kind: str | None = None) -> tuple[str, dict]:
    got = a.type_url.rsplit("/", 1)[-1]
    if kind is not None and got != kind:
        raise EnvelopeError(f"expected {kind}, got {got}")
    try:
        return got, json.loads(a.value.decode())
    except (UnicodeDecodeError, ValueError) as exc:
        raise EnvelopeError(f"bad {got} envelope: {exc}") from None


def _chunk_class():
    fdp = descriptor_pb2.FileDescriptorProto(name="swarm_b200_chunk.proto", package="swarm.v1",
                                             syntax="proto3")
    m = fdp.message_type.add(name="Chunk")
    F = descriptor_pb2.FieldDescriptorProto
    for i, (name, typ) in enumerate([("tensor_id", F.TYPE_STRING), ("chunk_index", F.TYPE_UINT32),
                                     ("chunk_count", F.TYPE_UINT32), ("total_length", F.TYPE_UINT64),
                                     ("payload", F.TYPE_BYTES), ("checksum", F.TYPE_STRING)], start=1):
        m.field.add(name=name, number=i, type=typ, label=F.LABEL_OPTIONAL)
    pool = descriptor_pool.DescriptorPool()
    pool.Add(fdp)
    return message_factory.GetMessageClass(pool.FindMessageTypeByName("swarm.v1.Chunk"))


Chunk = _chunk_class()


def to_chunks(tensor_id: str, data: bytes, chunk_bytes: int = CHUNK_BYTES):
    digest = hashlib.sha256(data).hexdigest()
    n = max(1, (len(data) + chunk_bytes - 1) // chunk_bytes)
    for i in range(n):
        yield Chunk(tensor_id=tensor_id, chunk_index=i, chunk_count=n, total_length=len(data),
                    payload=data[i * chunk_bytes:(i + 1) * chunk_bytes], checksum=digest)


class Reassembler:
    def __init__(self):
        self.parts: dict[str, dict[int, bytes]] = {}

    def add(self, c) -> tuple[str, bytes] | None:
        d = self.parts.setdefault(c.tensor_id, {})
        if c.chunk_index in d or c.chunk_index >= c.chunk_count:
            raise EnvelopeError(f"{c.tensor_id}: bad or duplicate chunk {c.chunk_index}")
        d[c.chunk_index] = bytes(c.payload)
        if len(d) < c.chunk_count:
            return None
        data = b"".join(d[i] for i in range(c.chunk_count))
        del self.parts[c.tensor_id]
        if len(data) != c.total_length or hashlib.sha256(data).hexdigest() != c.checksum:
            raise EnvelopeError(f"{c.tensor_id}: length or checksum mismatch")
        return c.tensor_id, data


COORDINATOR_METHODS = ("Register", "Heartbeat", "PlanModel", "DeployModel", "UnloadModel",
                       "TopologyStatus", "Workers", "Status", "PublishToken", "PairingCreate",
                       "CancelRequest", "SubmitStream")
WORKER_METHODS = ("Reserve", "Release", "HasArtifact", "FetchArtifact", "VerifyArtifact",
                  "LoadStage", "UnloadStage", "InstallRoute", "WithdrawRoute", "CheckPeer",
                  "FreeBytes", "Health")


class GrpcControlServer:
    """``handlers[(service, method)] = async fn(kind, obj) -> (kind, obj)``;
    ``server_streams[(service, method)] = async generator fn(kind, obj) -> (kind, obj)...``
    (server-streaming calls such as SubmitStream); ``stream_handler = async fn(tensor_id,
    data) -> bytes`` serves ExecuteStream.  While a handler runs, ``PEER_FINGERPRINT``
    holds the caller's certificate-bound identity fingerprint."""

    def __init__(self, handlers: dict, *, stream_handler=None, server_streams: dict | None = None,
                 host: str = "127.0.0.1", port: int = 0,
                 credentials: grpc.ServerCredentials | None = None):
        self.handlers = handlers
        self.stream_handler = stream_handler
        self.server_streams = server_streams or {}
        self.host, self.port = host, port
        self.creds = credentials
        self.server = None

    def _unary(self, fn):
        async def call(req, ctx):
            kind, obj = unpack(req)
            token = PEER_FINGERPRINT.set(_peer_fingerprint(ctx))
            try:
                rk, robj = await fn(kind, obj)
            except EnvelopeError as exc:
                await ctx.abort(grpc.StatusCode.INVALID_ARGUMENT, str(exc))
            except PermissionError as exc:
                await ctx.abort(grpc.StatusCode.PERMISSION_DENIED, str(exc))
            finally:
                PEER_FINGERPRINT.reset(token)
            return pack(rk, robj)
        return grpc.unary_unary_rpc_method_handler(
            call, request_deserializer=any_pb2.Any.FromString,
            response_serializer=any_pb2.Any.SerializeToString)

    def _server_stream(self, fn):
        async def call(req, ctx):
            kind, obj = unpack(req)
            token = PEER_FINGERPRINT.set(_peer_fingerprint(ctx))
            try:
                async for rk, robj in fn(kind, obj):
                    yield pack(rk, robj)
            except PermissionError as exc:
                await ctx.abort(grpc.StatusCode.PERMISSION_DENIED, str(exc))
            finally:
                PEER_FINGERPRINT.reset(token)
        return grpc.unary_stream_rpc_method_handler(
            call, request_deserializer=any_pb2.Any.FromString,
            response_serializer=any_pb2.Any.SerializeToString)

    def _stream(self):
        async def call(req_iter, ctx):
            ra = Reassembler()
            async for c in req_iter:
                try:
                    done = ra.add(c)
                except EnvelopeError as exc:
                    await ctx.abort(grpc.StatusCode.DATA_LOSS, str(exc))
                if done is not None:
                    out = await self.stream_handler(*done)
                    for oc in to_chunks(done[0] + ":out", out):
                        yield oc
        return grpc.stream_stream_rpc_method_handler(
            call, request_deserializer=Chunk.FromString, response_serializer=Chunk.SerializeToString)

    async def start(self) -> int:
        self.server = grpc.aio.server()
        by_service: dict[str, dict] = {}
        for (svc, method), fn in self.handlers.items():
            by_service.setdefault(svc, {})[method] = self._unary(fn)
        for (svc, method), fn in self.server_streams.items():
            by_service.setdefault(svc, {})[method] = self._server_stream(fn)
        if self.stream_handler is not None:
            by_service.setdefault("swarm.v1.Worker", {})["ExecuteStream"] = self._stream()
        for svc, methods in by_service.items():
            self.server.add_generic_rpc_handlers((grpc.method_handlers_generic_handler(svc, methods),))
        addr = f"{self.host}:{self.port}"
        self.port = (self.server.add_secure_port(addr, self.creds) if self.creds
                     else self.server.add_insecure_port(addr))
        await self.server.start()
        return self.port

    async def stop(self, grace: float = 0.5):
        if self.server is not None:
            await self.server.stop(grace)


class GrpcControlClient:
    def __init__(self, target: str, credentials: grpc.ChannelCredentials | None = None,
                 timeout: float = 30.0):
        self.channel = (grpc.aio.secure_channel(target, credentials) if credentials
                        else grpc.aio.insecure_channel(target))
        self.timeout = timeout

    async def call(self, service: str, method: str, kind: str, obj: dict,
                   expect: str | None = None) -> tuple[str, dict]:
        fn = self.channel.unary_unary(f"/{service}/{method}",
                                      request_serializer=any_pb2.Any.SerializeToString,
                                      response_deserializer=any_pb2.Any.FromString)
        rep = await fn(pack(kind, obj), timeout=self.timeout)
        return unpack(rep, expect)

    async def call_stream(self, service: str, method: str, kind: str, obj: dict,
                          timeout: float | None = None):
        """Server-streaming call: async iterator of (kind, obj) replies."""
        fn = self.channel.unary_stream(f"/{service}/{method}",
                                       request_serializer=any_pb2.Any.SerializeToString,
                                       response_deserializer=any_pb2.Any.FromString)
        async for rep in fn(pack(kind, obj), timeout=timeout):
            yield unpack(rep)

    async def execute_stream(self, tensor_id: str, data: bytes, chunk_bytes: int = CHUNK_BYTES) -> bytes:
        fn = self.channel.stream_stream("/swarm.v1.Worker/ExecuteStream",
                                        request_serializer=Chunk.SerializeToString,
                                        response_deserializer=Chunk.FromString)
        call = fn(iter(list(to_chunks(tensor_id, data, chunk_bytes))), timeout=self.timeout)
        ra = Reassembler()
        async for c in call:
            done = ra.add(c)
            if done is not None:
                return done[1]
        raise EnvelopeError("stream ended before the reply was complete")

    async def close(self):
        await self.channel.close()
