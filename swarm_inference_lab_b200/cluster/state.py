"""Cluster state store: versioned, atomically persisted security and runtime state.

Layout under the state root (default ``~/.swarm-b200``)::

    identity.json            node identity (Ed25519, 0600)
    cluster.json             cluster record: name, CA, coordinator endpoint/fingerprint,
                             members, revocations, pairing invitations (schema version)
    ca/ca.crt, ca/ca.key     cluster CA (coordinator only)
    tls/node.crt, node.key   this node's certificate
    runtime.json             ports, pids, deployments

Writes go through ``atomic_write``; ``_migrate`` upgrades older schema versions
in place.  Reference: si/cluster/state.py:62-853.
"""
from __future__ import annotations

import json
import time
from dataclasses import dataclass
from pathlib import Path

from ..coordinator.state import atomic_write
from ..security.identity import Identity

SCHEMA_VERSION = 2


class StateError(RuntimeError):
    pass


def _migrate(doc: dict) -> dict:
    v = doc.get("schema_version", 1)
    if v == 1:
        doc.setdefault("revoked", [])
        doc.setdefault("invitations", {})
        doc["schema_version"] = 2
    if doc["schema_version"] != SCHEMA_VERSION:
        raise StateError(f"unsupported cluster schema {doc['schema_version']}")
    return doc


@dataclass
class ClusterStateStore:
    root: Path

    def __post_init__(self):
        self.root = Path(self.root).expanduser()
        self.root.mkdir(parents=True, exist_ok=True)

    # identity
    def identity(self, name: str = "node") -> Identity:
        return Identity.load_or_create(self.root / "identity.json", name)

    # cluster record
    @property
    def cluster_path(self) -> Path:
        return self.root / "cluster.json"

    def has_cluster(self) -> bool:
        return self.cluster_path.exists()

    def load_cluster(self) -> dict:
        if not self.has_cluster():
            raise StateError(f"no cluster state under {self.root}; run `swarm cluster create` "
                             f"or `swarm node join` first")
        doc = _migrate(json.loads(self.cluster_path.read_text()))
        return doc

    def save_cluster(self, doc: dict) -> None:
        doc["schema_version"] = SCHEMA_VERSION
        doc["updated"] = time.time()
        atomic_write(self.cluster_path, doc)

    def create_cluster(self, name: str, coordinator_endpoint: str, ca_cert: bytes, ca_key: bytes) -> dict:
        if self.has_cluster():
            raise StateError("this node already belongs to a cluster")
        ident = self.identity("coordinator")
        (self.root / "ca").mkdir(exist_ok=True)
        (self.root / "ca" / "ca.crt").write_bytes(ca_cert)
        kp = self.root / "ca" / "ca.key"
        kp.write_bytes(ca_key)
        kp.chmod(0o600)
        doc = {"name": name, "role": "coordinator", "coordinator_endpoint": coordinator_endpoint,
               "coordinator_fingerprint": ident.fingerprint, "members": {}, "revoked": [],
               "invitations": {}, "created": time.time()}
        self.save_cluster(doc)
        return doc

    def ca(self) -> tuple[bytes, bytes | None]:
        crt = (self.root / "ca" / "ca.crt").read_bytes()
        key_p = self.root / "ca" / "ca.key"
        return crt, key_p.read_bytes() if key_p.exists() else None

    def save_node_tls(self, cert: bytes, key: bytes) -> None:
        (self.root / "tls").mkdir(exist_ok=True)
        (self.root / "tls" / "node.crt").write_bytes(cert)
        kp = self.root / "tls" / "node.key"
        kp.write_bytes(key)
        kp.chmod(0o600)

    def add_member(self, node_id: str, fingerprint: str, endpoint: str, caps: dict) -> None:
        doc = self.load_cluster()
        if fingerprint in doc["revoked"]:
            raise StateError("node identity is revoked")
        doc["members"][node_id] = {"fingerprint": fingerprint, "endpoint": endpoint,
                                   "capabilities": caps, "joined": time.time()}
        self.save_cluster(doc)

    def revoke(self, node_id: str) -> str:
        doc = self.load_cluster()
        m = doc["members"].pop(node_id, None)
        if m is None:
            raise StateError(f"unknown node {node_id}")
        doc["revoked"].append(m["fingerprint"])
        self.save_cluster(doc)
        return m["fingerprint"]

    # worker trust list: identities the coordinator admits at registration besides the
    # paired members (a revoked fingerprint stays refused)
    def trust(self, fingerprint: str, label: str = "", notes: str = "") -> bool:
        """Adds or updates a trusted worker fingerprint; True if it was new."""
        doc = self.load_cluster()
        if fingerprint in doc["revoked"]:
            raise StateError("node identity is revoked")
        trusted = doc.setdefault("trusted", {})
        added = fingerprint not in trusted
        trusted[fingerprint] = {"label": label, "notes": notes, "at": time.time()}
        self.save_cluster(doc)
        return added

    def untrust(self, fingerprint: str) -> bool:
        doc = self.load_cluster()
        gone = doc.setdefault("trusted", {}).pop(fingerprint, None) is not None
        self.save_cluster(doc)
        return gone

    def trusted(self) -> dict:
        return dict(self.load_cluster().get("trusted", {}))

    def delete(self) -> None:
        for p in sorted(self.root.rglob("*"), reverse=True):
            if p.is_file():
                p.unlink()
            elif p.is_dir():
                p.rmdir()

    # runtime
    def runtime(self) -> dict:
        p = self.root / "runtime.json"
        return json.loads(p.read_text()) if p.exists() else {}

    def save_runtime(self, doc: dict) -> None:
        atomic_write(self.root / "runtime.json", doc)
