"""Coordinator bookkeeping: durable state, per-request event streams and the worker registry.

* ``atomic_write`` / ``DurableState``: JSON state (requests, accepted tokens,
  replay tokens, workers, audit log) written via temp file + fsync + rename,
  so a crash leaves either the old or the new file.  ``mark_restart_boundaries``
  flags in-flight requests after a coordinator restart so they are replayed
  instead of silently resumed.
* ``EventStream``: bounded, strictly ordered per-request queue of events
  (TOKEN_GENERATED, REQUEST_COMPLETED, ...); sequence numbers are contiguous.
* ``WorkerRegistry``: capability records with heartbeat health; workers
  whose heartbeat is older than the timeout are marked unhealthy.

Reference: si/coordinator/durable_state.py:24-265, si/coordinator/event_stream.py:13,
si/coordinator/registry.py:27.
"""
from __future__ import annotations

import asyncio
import json
import os
import threading
import time
from dataclasses import asdict, dataclass, field
from pathlib import Path


def atomic_write(path: str | Path, data: dict) -> None:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_name(path.name + f".tmp{os.getpid()}")
    with open(tmp, "w") as f:
        json.dump(data, f, sort_keys=True)
        f.flush()
        os.fsync(f.fileno())
    os.replace(tmp, path)


class DurableState:
    def __init__(self, path: str | Path):
        self.path = Path(path)
        self._lock = threading.Lock()
        if self.path.exists():
            self.data = json.loads(self.path.read_text())
        else:
            self.data = {"version": 1, "requests": {}, "workers": {}, "audit": []}

    def _save(self):
        atomic_write(self.path, self.data)

    def record_request(self, request_id: str, prompt: list[int], params: dict) -> None:
        with self._lock:
            self.data["requests"][request_id] = {"prompt": prompt, "params": params,
                                                 "accepted": [], "state": "running",
                                                 "generation": 1, "created": time.time()}
            self._save()

    def accept_token(self, request_id: str, token: int) -> None:
        with self._lock:
            self.data["requests"][request_id]["accepted"].append(int(token))
            self._save()

    def set_state(self, request_id: str, state: str, **extra) -> None:
        with self._lock:
            self.data["requests"][request_id].update(state=state, **extra)
            self._save()

    def replay_tokens(self, request_id: str) -> list[int]:
        r = self.data["requests"][request_id]
        return list(r["prompt"]) + list(r["accepted"])

    def audit(self, event: str, **fields) -> None:
        with self._lock:
            self.data["audit"].append({"event": event, "ts": time.time(), **fields})
            self._save()

    def set_last_generation(self, generation: int) -> None:
        with self._lock:
            self.data["last_generation"] = max(int(generation),
                                               int(self.data.get("last_generation", 0)))
            self._save()

    def record_model(self, name: str, desc: dict) -> None:
        """A deployed model's description (model, stages, replicas, capacity), redeployed by
        a restarted coordinator."""
        with self._lock:
            self.data.setdefault("models", {})[name] = desc
            self._save()

    def drop_model(self, name: str) -> None:
        with self._lock:
            if self.data.setdefault("models", {}).pop(name, None) is not None:
                self._save()

    def models(self) -> dict:
        return dict(self.data.get("models", {}))

    def mark_restart_boundaries(self) -> list[str]:
        """After a restart: running requests become 'replay_required'."""
        with self._lock:
            hit = [rid for rid, r in self.data["requests"].items() if r["state"] == "running"]
            for rid in hit:
                self.data["requests"][rid]["state"] = "replay_required"
                self.data["requests"][rid]["generation"] += 1
            self._save()
            return hit


class EventStreamClosed(RuntimeError):
    pass


class EventStream:
    def __init__(self, request_id: str, maxsize: int = 4096):
        self.request_id = request_id
        self.queue: asyncio.Queue = asyncio.Queue(maxsize=maxsize)
        self.seq = 0
        self.closed = False

    async def put(self, kind: str, **payload) -> int:
        if self.closed:
            raise EventStreamClosed(self.request_id)
        self.seq += 1
        await self.queue.put({"seq": self.seq, "kind": kind, "request_id": self.request_id, **payload})
        if kind in ("REQUEST_COMPLETED", "REQUEST_FAILED", "REQUEST_CANCELLED"):
            self.closed = True
        return self.seq

    async def __aiter__(self):
        while True:
            ev = await self.queue.get()
            yield ev
            if ev["kind"] in ("REQUEST_COMPLETED", "REQUEST_FAILED", "REQUEST_CANCELLED"):
                return


@dataclass
class WorkerRecord:
    worker_id: str
    fingerprint: str
    endpoint: str
    capabilities: dict = field(default_factory=dict)
    last_heartbeat: float = field(default_factory=time.time)
    healthy: bool = True


class WorkerRegistry:
    def __init__(self, heartbeat_timeout_s: float = 15.0):
        self.timeout = heartbeat_timeout_s
        self.workers: dict[str, WorkerRecord] = {}

    def register(self, rec: WorkerRecord) -> None:
        rec.last_heartbeat = time.time()
        rec.healthy = True
        self.workers[rec.worker_id] = rec

    def heartbeat(self, worker_id: str, now: float | None = None) -> None:
        w = self.workers[worker_id]
        w.last_heartbeat = time.time() if now is None else now
        w.healthy = True

    def mark_unhealthy(self, worker_id: str) -> None:
        if worker_id in self.workers:
            self.workers[worker_id].healthy = False

    def sweep(self, now: float | None = None) -> list[str]:
        now = time.time() if now is None else now
        dead = [w.worker_id for w in self.workers.values()
                if w.healthy and now - w.last_heartbeat > self.timeout]
        for wid in dead:
            self.workers[wid].healthy = False
        return dead

    def healthy(self) -> list[WorkerRecord]:
        return [w for w in self.workers.values() if w.healthy]

    def snapshot(self) -> dict:
        return {k: asdict(v) for k, v in self.workers.items()}
