"""Single-use, transcript-bound node pairing.

The coordinator mints an invitation (random 256-bit secret, expiry, its
identity fingerprint and endpoint) rendered as a ``swarm-pair://`` URI.  A
joining node connects and both sides run an ephemeral X25519 exchange; the
session key is HKDF-SHA256(shared secret, salt = invitation secret, info =
transcript hash of both public keys and both identity fingerprints), so an
observer without the invitation learns nothing and a relayed exchange fails.
Each side proves possession of its Ed25519 identity by signing the
transcript; the node then sends its identity and capabilities under
AES-256-GCM and receives its TLS certificate and the cluster CA.  The
invitation is consumed on first use and rejected after expiry.

Reference: si/cluster/pairing.py:114-1079 (X25519 ECDH, AES-GCM, Ed25519
proofs, single-use invitations, certificate issue).
"""
from __future__ import annotations

import asyncio
import base64
import hashlib
import json
import os
import secrets
import time
from dataclasses import dataclass
from urllib.parse import parse_qs, urlparse

from cryptography.hazmat.primitives import hashes, serialization
from cryptography.hazmat.primitives.asymmetric.x25519 import X25519PrivateKey, X25519PublicKey
from cryptography.hazmat.primitives.ciphers.aead import AESGCM
from cryptography.hazmat.primitives.kdf.hkdf import HKDF

from ..security.identity import SignatureError, canonical, fingerprint, public_key
from ..security.tls import issue_node_cert
from .state import ClusterStateStore


class PairingError(RuntimeError):
    pass


def _b64(b: bytes) -> str:
    return base64.b64encode(b).decode()


def _unb64(s: str) -> bytes:
    return base64.b64decode(s)


@dataclass
class Invitation:
    token: str
    endpoint: str
    coordinator_fingerprint: str
    expires_at: float

    def uri(self) -> str:
        host, port = self.endpoint.rsplit(":", 1)
        return (f"swarm-pair://{host}:{port}/?token={self.token}"
                f"&fp={self.coordinator_fingerprint}&exp={int(self.expires_at)}")

    @classmethod
    def parse(cls, uri: str) -> "Invitation":
        u = urlparse(uri)
        if u.scheme != "swarm-pair":
            raise PairingError("not a swarm-pair:// URI")
        q = parse_qs(u.query)
        return cls(q["token"][0], f"{u.hostname}:{u.port}", q["fp"][0], float(q["exp"][0]))


def _session_key(shared: bytes, token: str, transcript: bytes) -> bytes:
    return HKDF(algorithm=hashes.SHA256(), length=32, salt=bytes.fromhex(token),
                info=b"swarm-b200-pairing" + transcript).derive(shared)


def _transcript(coord_pub: bytes, node_pub: bytes, coord_fp: str, node_fp: str) -> bytes:
    return hashlib.sha256(coord_pub + node_pub + coord_fp.encode() + node_fp.encode()).digest()


async def _send(w, obj):
    w.write(json.dumps(obj).encode() + b"\n")
    await w.drain()


async def _recv(r, timeout=30.0):
    line = await asyncio.wait_for(r.readline(), timeout)
    if not line:
        raise PairingError("peer closed the pairing connection")
    return json.loads(line)


class PairingManager:
    """Coordinator side: invitations and the pairing server."""

    def __init__(self, store: ClusterStateStore, endpoint: str):
        self.store = store
        self.endpoint = endpoint
        self.ident = store.identity("coordinator")
        self.server = None
        self._tokens: dict[str, str] = {}  # invitation hash -> secret (memory only)

    def invite(self, ttl_s: float = 600.0) -> Invitation:
        doc = self.store.load_cluster()
        inv = Invitation(secrets.token_hex(32), self.endpoint, self.ident.fingerprint,
                         time.time() + ttl_s)
        h = hashlib.sha256(inv.token.encode()).hexdigest()
        doc["invitations"][h] = {"expires_at": inv.expires_at, "used": False}
        self._tokens[h] = inv.token
        self.store.save_cluster(doc)
        return inv

    def _consume(self, token: str) -> None:
        doc = self.store.load_cluster()
        key = hashlib.sha256(token.encode()).hexdigest()
        rec = doc["invitations"].get(key)
        if rec is None:
            raise PairingError("unknown invitation")
        if rec["used"]:
            raise PairingError("invitation already used")
        if rec["expires_at"] < time.time():
            raise PairingError("invitation expired")
        rec["used"] = True
        self.store.save_cluster(doc)

    async def start(self, host: str = "127.0.0.1", port: int = 0) -> int:
        self.server = await asyncio.start_server(self._serve, host, port)
        return self.server.sockets[0].getsockname()[1]

    async def _serve(self, r, w):
        try:
            hello = await _recv(r)
            eph = X25519PrivateKey.generate()
            cpub = eph.public_key().public_bytes(serialization.Encoding.Raw, serialization.PublicFormat.Raw)
            npub = _unb64(hello["x25519"])
            tr = _transcript(cpub, npub, self.ident.fingerprint, hello["fingerprint"])
            await _send(w, {"x25519": _b64(cpub), "fingerprint": self.ident.fingerprint,
                            "identity_key": _b64(self.ident.public_raw), "proof": self.ident.sign(tr)})
            sealed = await _recv(r)
            # The token is known only to holders of the invitation: try the unused ones.
            doc = self.store.load_cluster()
            shared = eph.exchange(X25519PublicKey.from_public_bytes(npub))
            body = None
            hint = sealed.get("invitation")  # SHA-256 of the secret; the secret never travels
            rec = doc["invitations"].get(hint)
            token = self._tokens.get(hint)
            if rec is not None and token is not None and not rec["used"]:
                k = _session_key(shared, token, tr)
                body = json.loads(AESGCM(k).decrypt(_unb64(sealed["nonce"]), _unb64(sealed["ct"]), tr))
                self._consume(token)
            if body is None:
                raise PairingError("no matching invitation")
            node_key = _unb64(body["identity_key"])
            if fingerprint(node_key) != hello["fingerprint"]:
                raise PairingError("node identity does not match its fingerprint")
            try:
                public_key(node_key).verify(_unb64(body["proof"]), tr)
            except Exception:
                raise PairingError("node proof of possession failed") from None
            ca_crt, ca_key = self.store.ca()
            from ..security.tls import PemPair
            cert = issue_node_cert(PemPair(ca_crt, ca_key), body["node_id"], hello["fingerprint"],
                                   body.get("hosts", ["127.0.0.1"]))
            self.store.add_member(body["node_id"], hello["fingerprint"], body.get("endpoint", ""),
                                  body.get("capabilities", {}))
            reply = {"cert": cert.cert.decode(), "key": cert.key.decode(), "ca": ca_crt.decode(),
                     "cluster": doc["name"], "coordinator_endpoint": doc["coordinator_endpoint"]}
            nonce = os.urandom(12)
            await _send(w, {"nonce": _b64(nonce), "ct": _b64(AESGCM(k).encrypt(nonce, canonical(reply), tr))})
        except (PairingError, SignatureError, KeyError, ValueError) as exc:
            try:
                await _send(w, {"error": str(exc)})
            except Exception:  # noqa: BLE001
                pass
        finally:
            w.close()

    async def close(self):
        if self.server:
            self.server.close()
            await self.server.wait_closed()


async def join(uri: str, store: ClusterStateStore, node_id: str, *, capabilities: dict | None = None,
               endpoint: str = "", hosts: list[str] | None = None) -> dict:
    """Node side: pair with the coordinator named by ``uri``; stores cert + CA + cluster record."""
    inv = Invitation.parse(uri)
    if inv.expires_at < time.time():
        raise PairingError("invitation expired")
    ident = store.identity(node_id)
    host, port = inv.endpoint.rsplit(":", 1)
    r, w = await asyncio.open_connection(host, int(port))
    try:
        eph = X25519PrivateKey.generate()
        npub = eph.public_key().public_bytes(serialization.Encoding.Raw, serialization.PublicFormat.Raw)
        await _send(w, {"x25519": _b64(npub), "fingerprint": ident.fingerprint})
        rep = await _recv(r)
        if "error" in rep:
            raise PairingError(rep["error"])
        if rep["fingerprint"] != inv.coordinator_fingerprint:
            raise PairingError("coordinator fingerprint does not match the invitation")
        ckey = _unb64(rep["identity_key"])
        if fingerprint(ckey) != rep["fingerprint"]:
            raise PairingError("coordinator key does not match its fingerprint")
        cpub = _unb64(rep["x25519"])
        tr = _transcript(cpub, npub, rep["fingerprint"], ident.fingerprint)
        try:
            public_key(ckey).verify(_unb64(rep["proof"]), tr)
        except Exception:
            raise PairingError("coordinator proof of possession failed") from None
        k = _session_key(eph.exchange(X25519PublicKey.from_public_bytes(cpub)), inv.token, tr)
        body = {"node_id": node_id, "identity_key": _b64(ident.public_raw),
                "proof": ident.sign(tr), "capabilities": capabilities or {}, "endpoint": endpoint,
                "hosts": hosts or ["127.0.0.1"]}
        nonce = os.urandom(12)
        await _send(w, {"invitation": hashlib.sha256(inv.token.encode()).hexdigest(),
                        "nonce": _b64(nonce),
                        "ct": _b64(AESGCM(k).encrypt(nonce, canonical(body), tr))})
        fin = await _recv(r)
        if "error" in fin:
            raise PairingError(fin["error"])
        reply = json.loads(AESGCM(k).decrypt(_unb64(fin["nonce"]), _unb64(fin["ct"]), tr))
    finally:
        w.close()
    store.save_node_tls(reply["cert"].encode(), reply["key"].encode())
    (store.root / "ca").mkdir(exist_ok=True)
    (store.root / "ca" / "ca.crt").write_bytes(reply["ca"].encode())
    store.save_cluster({"name": reply["cluster"], "role": "node",
                        "coordinator_endpoint": reply["coordinator_endpoint"],
                        "coordinator_fingerprint": inv.coordinator_fingerprint, "members": {},
                        "revoked": [], "invitations": {}, "node_id": node_id})
    return reply
