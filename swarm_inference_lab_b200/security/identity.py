"""Node identities (Ed25519), canonical-JSON signatures and signed route leases.

* ``Identity``: a versioned Ed25519 key pair persisted with 0600 permissions;
  its fingerprint is the SHA-256 of the raw public key.
* ``sign_record`` / ``verify_record``: signatures over canonical JSON
  (sorted keys, compact separators) so any party can re-derive the bytes.
* ``RouteLease``: the coordinator-signed, finite-lived authorisation a stage
  owner checks before installing a route: topology, route generation, model
  and tokenizer revisions, ordered stage assignments with worker
  fingerprints and endpoints, issue/expiry time and a one-time nonce.
  ``LeaseVerifier`` rejects unknown signers, bad signatures, expired or
  future-dated leases, reused nonces and stale generations.

Reference: si/security/identity.py:111-303, si/security/signatures.py:15-30,
si/protocol/routes.py:114-322 (signed route leases and verification rules).
"""
from __future__ import annotations

import base64
import hashlib
import json
import os
import secrets
import time
from dataclasses import asdict, dataclass, field
from pathlib import Path

from cryptography.exceptions import InvalidSignature
from cryptography.hazmat.primitives import serialization
from cryptography.hazmat.primitives.asymmetric.ed25519 import Ed25519PrivateKey, Ed25519PublicKey

IDENTITY_VERSION = 1


class SignatureError(ValueError):
    pass


def canonical(obj) -> bytes:
    return json.dumps(obj, sort_keys=True, separators=(",", ":"), ensure_ascii=False,
                      allow_nan=False).encode()


def fingerprint(public_raw: bytes) -> str:
    return "sha256:" + hashlib.sha256(public_raw).hexdigest()


@dataclass
class Identity:
    name: str
    key: Ed25519PrivateKey
    version: int = IDENTITY_VERSION

    @classmethod
    def generate(cls, name: str) -> "Identity":
        return cls(name, Ed25519PrivateKey.generate())

    @property
    def public_raw(self) -> bytes:
        return self.key.public_key().public_bytes(serialization.Encoding.Raw,
                                                   serialization.PublicFormat.Raw)

    @property
    def fingerprint(self) -> str:
        return fingerprint(self.public_raw)

    def sign(self, data: bytes) -> str:
        return base64.b64encode(self.key.sign(data)).decode()

    def save(self, path: str | Path) -> None:
        path = Path(path)
        path.parent.mkdir(parents=True, exist_ok=True)
        raw = self.key.private_bytes(serialization.Encoding.Raw, serialization.PrivateFormat.Raw,
                                     serialization.NoEncryption())
        doc = {"version": self.version, "name": self.name,
               "private_key": base64.b64encode(raw).decode(), "fingerprint": self.fingerprint}
        tmp = path.with_suffix(".tmp")
        fd = os.open(tmp, os.O_WRONLY | os.O_CREAT | os.O_TRUNC, 0o600)
        with os.fdopen(fd, "w") as f:
            json.dump(doc, f)
        os.replace(tmp, path)

    @classmethod
    def load(cls, path: str | Path) -> "Identity":
        doc = json.loads(Path(path).read_text())
        if doc.get("version") != IDENTITY_VERSION:
            raise SignatureError(f"unsupported identity version {doc.get('version')}")
        key = Ed25519PrivateKey.from_private_bytes(base64.b64decode(doc["private_key"]))
        ident = cls(doc["name"], key)
        if ident.fingerprint != doc["fingerprint"]:
            raise SignatureError("identity file fingerprint does not match its key")
        return ident

    @classmethod
    def load_or_create(cls, path: str | Path, name: str) -> "Identity":
        p = Path(path)
        if p.exists():
            return cls.load(p)
        ident = cls.generate(name)
        ident.save(p)
        return ident


def public_key(raw: bytes) -> Ed25519PublicKey:
    return Ed25519PublicKey.from_public_bytes(raw)


def sign_record(ident: Identity, record: dict) -> dict:
    body = {k: v for k, v in record.items() if k != "signature"}
    body["signer"] = ident.fingerprint
    body["signer_key"] = base64.b64encode(ident.public_raw).decode()
    body["signature"] = ident.sign(canonical(body))
    return body


def verify_record(record: dict, trusted: set[str] | None = None) -> dict:
    try:
        sig = base64.b64decode(record["signature"])
        raw = base64.b64decode(record["signer_key"])
    except (KeyError, ValueError) as exc:
        raise SignatureError(f"unsigned or malformed record: {exc}") from None
    if fingerprint(raw) != record.get("signer"):
        raise SignatureError("signer fingerprint does not match the embedded key")
    if trusted is not None and record["signer"] not in trusted:
        raise SignatureError("record signed by an untrusted identity")
    body = {k: v for k, v in record.items() if k != "signature"}
    try:
        public_key(raw).verify(sig, canonical(body))
    except InvalidSignature:
        raise SignatureError("bad signature") from None
    return body


@dataclass
class StageAssignment:
    stage_id: int
    worker_id: str
    worker_fingerprint: str
    layer_start: int
    layer_end: int
    control_endpoint: str
    data_endpoint: str


@dataclass
class RouteLease:
    topology_id: str
    generation: int
    model_revision: str
    tokenizer_revision: str
    adapter: str
    dtype: str
    stages: list[StageAssignment]
    issued_at: float = field(default_factory=time.time)
    expires_at: float = 0.0
    nonce: str = field(default_factory=lambda: secrets.token_hex(16))

    def record(self) -> dict:
        d = asdict(self)
        d["kind"] = "route_lease"
        return d

    @classmethod
    def from_record(cls, d: dict) -> "RouteLease":
        d = {k: v for k, v in d.items() if k in cls.__dataclass_fields__}
        d["stages"] = [StageAssignment(**s) for s in d["stages"]]
        return cls(**d)


def issue_lease(coordinator: Identity, lease: RouteLease, ttl_s: float = 300.0) -> dict:
    if not lease.expires_at:
        lease.expires_at = lease.issued_at + ttl_s
    return sign_record(coordinator, lease.record())


class LeaseVerifier:
    def __init__(self, coordinator_fingerprint: str, *, max_future_s: float = 30.0,
                 nonce_cache: int = 4096):
        self.coordinator = coordinator_fingerprint
        self.max_future = max_future_s
        self.nonces: list[str] = []
        self.cache = nonce_cache
        self.generation = -1

    def verify(self, signed: dict, *, now: float | None = None, worker_fingerprint: str | None = None,
               model_revision: str | None = None) -> RouteLease:
        body = verify_record(signed, {self.coordinator})
        if body.get("kind") != "route_lease":
            raise SignatureError("not a route lease")
        lease = RouteLease.from_record(body)
        now = time.time() if now is None else now
        if lease.expires_at <= now:
            raise SignatureError("lease expired")
        if lease.issued_at > now + self.max_future:
            raise SignatureError("lease issued in the future")
        if lease.nonce in self.nonces:
            raise SignatureError("lease nonce reused")
        if lease.generation <= self.generation:
            raise SignatureError(f"stale route generation {lease.generation} <= {self.generation}")
        if worker_fingerprint and not any(s.worker_fingerprint == worker_fingerprint for s in lease.stages):
            raise SignatureError("lease does not assign this worker")
        if model_revision and lease.model_revision != model_revision:
            raise SignatureError("lease is for another model revision")
        self.nonces.append(lease.nonce)
        del self.nonces[:-self.cache]
        self.generation = lease.generation
        return lease
