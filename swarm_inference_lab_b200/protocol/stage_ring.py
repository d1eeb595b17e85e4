"""SWRING01 stage-ring frames: codec, limits and per-edge sequence validation.

Frame = 76-byte little-endian header ``<8sHHIIQQihh32s`` | canonical JSON
metadata | opaque payload.  Header fields: magic ``SWRING01``, version (1),
operation, flags, metadata length, payload length, sequence number, token
position, source stage, destination stage, SHA-256 of metadata || payload.

The header layout, operation codes, metadata keys and limits are kept
identical to the reference protocol (docs/stage-ring-protocol.md,
si/protocol/stage_ring.py:29-51, 162-207) so frames interoperate with its
stage owners; the encoder/decoder below and the C++ codec in
``csrc/native/stage_ring.cpp`` are independent implementations that share
golden vectors in the tests.
"""
from __future__ import annotations

import enum
import hashlib
import hmac
import json
import math
import struct
from dataclasses import dataclass, field
from typing import Any

MAGIC = b"SWRING01"
VERSION = 1
HEADER = struct.Struct("<8sHHIIQQihh32s")
HEADER_SIZE = HEADER.size  # 76
MAX_METADATA = 4 * 1024 * 1024
MAX_PAYLOAD = 1024 * 1024 * 1024
COORDINATOR = -1


class Operation(enum.IntEnum):
    HELLO = 1
    CAPABILITIES = 2
    LOAD_STAGE = 3
    OPEN_SESSION = 4
    PREFILL = 5
    DECODE = 6
    VERIFY_CANDIDATES = 7
    TOKEN_RESULT = 8
    SESSION_CHECKPOINT = 9
    CLOSE_SESSION = 10
    CANCEL_SESSION = 11
    HEALTH = 12
    ERROR = 13


class FrameError(ValueError):
    """A frame violated the wire format, limits or checksum."""


class SequenceError(ValueError):
    """A frame arrived duplicated, stale or after a gap on its session edge."""


class SessionError(ValueError):
    """A frame referenced an unknown, closed or mismatched session."""


METADATA_KEYS = (
    "attributes", "compression_mode", "destination_stage", "layer_range", "message_type",
    "model_revision", "payload_length", "protocol_version", "request_id", "sequence_number",
    "session_id", "source_stage", "stage_id", "stage_topology_id", "status", "tensor_dtype",
    "tensor_shape", "token_position", "tokenizer_revision",
)


@dataclass
class StageMessage:
    operation: Operation
    model_revision: str
    tokenizer_revision: str
    topology_id: str
    stage_id: int
    layer_start: int
    layer_end: int
    session_id: str
    request_id: str
    sequence_number: int
    token_position: int
    source_stage: int
    destination_stage: int
    tensor_shape: tuple[int, ...] = ()
    tensor_dtype: str = "none"
    compression_mode: str = "none"
    payload: bytes = b""
    status: str = "OK"
    flags: int = 0
    attributes: dict[str, Any] = field(default_factory=dict)

    def metadata(self) -> dict[str, Any]:
        return {
            "protocol_version": VERSION,
            "model_revision": self.model_revision,
            "tokenizer_revision": self.tokenizer_revision,
            "stage_topology_id": self.topology_id,
            "stage_id": self.stage_id,
            "layer_range": [self.layer_start, self.layer_end],
            "session_id": self.session_id,
            "request_id": self.request_id,
            "sequence_number": self.sequence_number,
            "token_position": self.token_position,
            "source_stage": self.source_stage,
            "destination_stage": self.destination_stage,
            "message_type": self.operation.name,
            "tensor_shape": list(self.tensor_shape),
            "tensor_dtype": self.tensor_dtype,
            "compression_mode": self.compression_mode,
            "payload_length": len(self.payload),
            "status": self.status,
            "attributes": self.attributes,
        }


def canonical_json(obj: Any) -> bytes:
    """Sorted keys, compact separators, UTF-8, no NaN/inf."""
    return json.dumps(obj, sort_keys=True, separators=(",", ":"), ensure_ascii=False,
                      allow_nan=False).encode("utf-8")


@dataclass(frozen=True)
class FrameHeader:
    operation: Operation
    flags: int
    metadata_length: int
    payload_length: int
    sequence_number: int
    token_position: int
    source_stage: int
    destination_stage: int
    checksum: bytes

    @property
    def body_length(self) -> int:
        return self.metadata_length + self.payload_length


def _check_stage(v: int, name: str, allow_coordinator: bool) -> None:
    lo = -1 if allow_coordinator else 0
    if not isinstance(v, int) or isinstance(v, bool) or not lo <= v <= 32767:
        raise FrameError(f"{name} out of range: {v!r}")


def encode(msg: StageMessage) -> bytes:
    """Serialize one message into a complete frame."""
    if not isinstance(msg.operation, Operation):
        raise FrameError("unknown operation")
    _check_stage(msg.source_stage, "source_stage", True)
    _check_stage(msg.destination_stage, "destination_stage", True)
    _check_stage(msg.stage_id, "stage_id", True)
    if not 0 <= msg.sequence_number < 2 ** 64:
        raise FrameError("sequence number out of range")
    if not -1 <= msg.token_position < 2 ** 31:
        raise FrameError("token position out of range")
    meta = canonical_json(msg.metadata())
    payload = bytes(msg.payload)
    if len(meta) > MAX_METADATA:
        raise FrameError("metadata exceeds 4 MiB")
    if len(payload) > MAX_PAYLOAD:
        raise FrameError("payload exceeds 1 GiB")
    digest = hashlib.sha256(meta + payload).digest()
    head = HEADER.pack(MAGIC, VERSION, int(msg.operation), msg.flags & 0xFFFFFFFF, len(meta),
                       len(payload), msg.sequence_number, msg.token_position, msg.source_stage,
                       msg.destination_stage, digest)
    return head + meta + payload


def decode_header(buf: bytes) -> FrameHeader:
    if len(buf) < HEADER_SIZE:
        raise FrameError("short header")
    magic, ver, op, flags, mlen, plen, seq, pos, src, dst, digest = HEADER.unpack_from(buf)
    if magic != MAGIC:
        raise FrameError("bad magic")
    if ver != VERSION:
        raise FrameError(f"unsupported version {ver}")
    try:
        operation = Operation(op)
    except ValueError:
        raise FrameError(f"unknown operation code {op}") from None
    if mlen > MAX_METADATA:
        raise FrameError("metadata exceeds 4 MiB")
    if plen > MAX_PAYLOAD:
        raise FrameError("payload exceeds 1 GiB")
    _check_stage(src, "source_stage", True)
    _check_stage(dst, "destination_stage", True)
    if pos < -1:
        raise FrameError("token position out of range")
    return FrameHeader(operation, flags, mlen, plen, seq, pos, src, dst, digest)


def decode_body(header: FrameHeader, body: bytes | memoryview) -> StageMessage:
    if len(body) != header.body_length:
        raise FrameError("declared and actual lengths differ")
    body = bytes(body)
    meta_b = body[: header.metadata_length]
    payload = body[header.metadata_length:]
    if not hmac.compare_digest(hashlib.sha256(body).digest(), header.checksum):
        raise FrameError("checksum mismatch")
    try:
        meta = json.loads(meta_b.decode("utf-8"),
                          parse_constant=lambda c: (_ for _ in ()).throw(FrameError(c)))
    except (UnicodeDecodeError, json.JSONDecodeError) as exc:
        raise FrameError(f"malformed metadata: {exc}") from None
    if not isinstance(meta, dict) or tuple(sorted(meta)) != METADATA_KEYS:
        raise FrameError("metadata keys missing, unknown or duplicated")
    if canonical_json(meta) != meta_b:
        raise FrameError("metadata is not canonical JSON")
    checks = {
        "protocol_version": VERSION,
        "message_type": header.operation.name,
        "sequence_number": header.sequence_number,
        "token_position": header.token_position,
        "source_stage": header.source_stage,
        "destination_stage": header.destination_stage,
        "payload_length": header.payload_length,
    }
    for k, v in checks.items():
        if meta[k] != v or isinstance(meta[k], bool):
            raise FrameError(f"header/metadata disagree on {k}")
    lr = meta["layer_range"]
    if not (isinstance(lr, list) and len(lr) == 2 and all(isinstance(x, int) for x in lr)):
        raise FrameError("layer_range malformed")
    shape = meta["tensor_shape"]
    if not isinstance(shape, list) or not all(isinstance(x, int) and x >= 0 for x in shape):
        raise FrameError("tensor_shape malformed")
    if not isinstance(meta["attributes"], dict):
        raise FrameError("attributes must be an object")
    for k in ("model_revision", "tokenizer_revision", "stage_topology_id", "session_id",
              "request_id", "tensor_dtype", "compression_mode", "status"):
        if not isinstance(meta[k], str):
            raise FrameError(f"{k} must be a string")
    _check_stage(meta["stage_id"], "stage_id", True)
    return StageMessage(
        operation=header.operation, model_revision=meta["model_revision"],
        tokenizer_revision=meta["tokenizer_revision"], topology_id=meta["stage_topology_id"],
        stage_id=meta["stage_id"], layer_start=lr[0], layer_end=lr[1],
        session_id=meta["session_id"], request_id=meta["request_id"],
        sequence_number=header.sequence_number, token_position=header.token_position,
        source_stage=header.source_stage, destination_stage=header.destination_stage,
        tensor_shape=tuple(shape), tensor_dtype=meta["tensor_dtype"],
        compression_mode=meta["compression_mode"], payload=payload, status=meta["status"],
        flags=header.flags, attributes=meta["attributes"])


def decode(frame: bytes) -> StageMessage:
    h = decode_header(frame[:HEADER_SIZE])
    return decode_body(h, frame[HEADER_SIZE:])


# --------------------------------------------------------------- validators
class SequenceValidator:
    """Strict +1 sequence numbers per (session, source, destination) edge."""

    def __init__(self):
        self._last: dict[tuple[str, int, int], int] = {}

    def check(self, msg: StageMessage) -> None:
        key = (msg.session_id, msg.source_stage, msg.destination_stage)
        prev = self._last.get(key)
        seq = msg.sequence_number
        if prev is not None:
            if seq == prev:
                raise SequenceError(f"duplicate sequence {seq} on {key}")
            if seq < prev:
                raise SequenceError(f"stale sequence {seq} < {prev} on {key}")
            if seq != prev + 1:
                raise SequenceError(f"sequence gap {prev} -> {seq} on {key}")
        self._last[key] = seq

    def reset_session(self, session_id: str) -> None:
        for k in [k for k in self._last if k[0] == session_id]:
            del self._last[k]


class SequenceAllocator:
    """Next sequence number per edge (sender side)."""

    def __init__(self):
        self._next: dict[tuple[str, int, int], int] = {}

    def next(self, session_id: str, src: int, dst: int) -> int:
        key = (session_id, src, dst)
        n = self._next.get(key, 0)
        self._next[key] = n + 1
        return n

    def reset_session(self, session_id: str) -> None:
        for k in [k for k in self._next if k[0] == session_id]:
            del self._next[k]


@dataclass
class SessionPin:
    model_revision: str
    topology_id: str
    tokenizer_revision: str | None = None
    stage_id: int | None = None
    layer_range: tuple[int, int] | None = None


SESSIONLESS = {Operation.HELLO, Operation.CAPABILITIES, Operation.LOAD_STAGE, Operation.HEALTH,
               Operation.ERROR}


class SessionValidator:
    """Open-once sessions pinned to model revision, topology and stage interval."""

    def __init__(self, pin: SessionPin):
        self.pin = pin
        self.active: set[str] = set()
        self.closed: set[str] = set()

    def check(self, msg: StageMessage) -> None:
        p = self.pin
        if msg.model_revision != p.model_revision:
            raise SessionError("model revision mismatch")
        if msg.topology_id != p.topology_id:
            raise SessionError("topology mismatch")
        if p.tokenizer_revision is not None and msg.tokenizer_revision != p.tokenizer_revision:
            raise SessionError("tokenizer revision mismatch")
        if p.stage_id is not None and msg.destination_stage not in (p.stage_id, COORDINATOR):
            raise SessionError("frame addressed to another stage")
        if p.layer_range is not None and msg.operation in (Operation.PREFILL, Operation.DECODE,
                                                           Operation.VERIFY_CANDIDATES):
            if (msg.layer_start, msg.layer_end) != tuple(p.layer_range):
                raise SessionError("layer interval mismatch")
        op = msg.operation
        if op in SESSIONLESS and not msg.session_id:
            return
        if op == Operation.OPEN_SESSION:
            if not msg.session_id:
                raise SessionError("empty session id")
            if msg.session_id in self.active or msg.session_id in self.closed:
                raise SessionError(f"session {msg.session_id} opened twice")
            self.active.add(msg.session_id)
            return
        if msg.session_id not in self.active:
            raise SessionError(f"session {msg.session_id!r} is not active")
        if op in (Operation.CLOSE_SESSION, Operation.CANCEL_SESSION):
            self.active.discard(msg.session_id)
            self.closed.add(msg.session_id)


def is_finite_json(obj: Any) -> bool:
    if isinstance(obj, float):
        return math.isfinite(obj)
    if isinstance(obj, dict):
        return all(is_finite_json(v) for v in obj.values())
    if isinstance(obj, list):
        return all(is_finite_json(v) for v in obj)
    return True
