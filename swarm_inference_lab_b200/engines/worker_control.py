"""Coordinator-authorised engine leases for worker-owned engines.

A worker starts or stops an engine process (an external or native engine it
owns) only when the coordinator hands it a signed engine lease naming the
worker's fingerprint, the engine, the model revision and an expiry; leases are
single-use (nonce) and a newer lease generation supersedes older ones.  The
controller keeps the running engines and stops those whose lease expired.

Reference: si/engines/worker_control.py:93; si/protocol/engine_worker.py:31-120;
si/worker/engine_runtime.py:30.
"""
from __future__ import annotations

import secrets
import time
from dataclasses import dataclass

from ..security.identity import Identity, SignatureError, sign_record, verify_record


def issue_engine_lease(coordinator: Identity, *, worker_fingerprint: str, engine: str,
                       model_revision: str, generation: int, action: str = "start",
                       ttl_s: float = 600.0) -> dict:
    return sign_record(coordinator, {"kind": "engine_lease", "worker": worker_fingerprint,
                                     "engine": engine, "model_revision": model_revision,
                                     "generation": int(generation), "action": action,
                                     "nonce": secrets.token_hex(12), "expires_at": time.time() + ttl_s})


@dataclass
class RunningEngine:
    engine: str
    model_revision: str
    generation: int
    expires_at: float
    handle: object


class EngineController:
    def __init__(self, worker_fingerprint: str, coordinator_fingerprint: str, launch, *, clock=time.time):
        self.me = worker_fingerprint
        self.trusted = {coordinator_fingerprint}
        self.launch = launch          # (engine, model_revision) -> handle with .stop()
        self.clock = clock
        self.running: dict[str, RunningEngine] = {}
        self._nonces: set[str] = set()
        self._generation = -1

    def _verify(self, signed: dict) -> dict:
        body = verify_record(signed, self.trusted)
        if body.get("kind") != "engine_lease" or body.get("worker") != self.me:
            raise SignatureError("lease is not for this worker")
        if body["expires_at"] <= self.clock():
            raise SignatureError("lease expired")
        if body["nonce"] in self._nonces:
            raise SignatureError("lease replayed")
        if body["generation"] < self._generation:
            raise SignatureError("stale lease generation")
        self._nonces.add(body["nonce"])
        self._generation = body["generation"]
        return body

    def apply(self, signed: dict) -> str:
        b = self._verify(signed)
        name = b["engine"]
        if b["action"] == "stop":
            r = self.running.pop(name, None)
            if r is not None:
                r.handle.stop()
            return "stopped"
        if name in self.running:
            self.running[name].handle.stop()
        self.running[name] = RunningEngine(name, b["model_revision"], b["generation"], b["expires_at"],
                                           self.launch(name, b["model_revision"]))
        return "started"

    def sweep(self) -> list[str]:
        now = self.clock()
        gone = [n for n, r in self.running.items() if r.expires_at <= now]
        for n in gone:
            self.running.pop(n).handle.stop()
        return gone
