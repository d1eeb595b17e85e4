"""Multi-process loopback harness: stage workers as real OS processes.

``ManagedProcess`` spawns a worker, waits for its ready line with a bounded
timeout, and kills it (bounded) on stop; every started process is tracked so
tests can assert that none leaked.  ``LoopbackRing`` starts an N-stage ring
(last stage first so each upstream stage knows its next hop), exposes the
route for a :class:`~swarm_inference_lab_b200.coordinator.session.SessionController`,
and implements restart-and-reinstall recovery: dead workers are restarted
and every stage receives the next route generation.

Reference: si/testing/process_harness.py:61-443 (``ManagedProcess``,
``ProductCluster``) and the stage-ring integration fixtures in
tests/integration/test_product_stage_ring.py.
"""
from __future__ import annotations

import asyncio
import json
import os
import subprocess
import sys
import time
from dataclasses import dataclass, field

from ..protocol import stage_ring as sr
from ..transport.stage_ring_net import StageRingConnection

LIVE: set[int] = set()  # pids started by this module and not yet reaped


class ManagedProcess:
    def __init__(self, args: list[str], *, ready_timeout: float = 120.0, env: dict | None = None):
        self.args = args
        self.ready_timeout = ready_timeout
        self.env = env
        self.proc: subprocess.Popen | None = None
        self.ready: dict = {}

    def start(self) -> dict:
        env = dict(os.environ)
        env.update(self.env or {})
        root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        env["PYTHONPATH"] = root + os.pathsep + env.get("PYTHONPATH", "")
        self.proc = subprocess.Popen([sys.executable, *self.args], stdout=subprocess.PIPE,
                                     stderr=subprocess.PIPE, env=env, text=True)
        LIVE.add(self.proc.pid)
        deadline = time.monotonic() + self.ready_timeout
        import selectors
        sel = selectors.DefaultSelector()
        sel.register(self.proc.stdout, selectors.EVENT_READ)
        while time.monotonic() < deadline:
            if self.proc.poll() is not None:
                err = self.proc.stderr.read()
                self.stop()
                raise RuntimeError(f"worker exited before ready: {err[-2000:]}")
            if sel.select(timeout=0.2):
                line = self.proc.stdout.readline()
                if line.startswith("{"):
                    self.ready = json.loads(line)
                    sel.close()
                    return self.ready
        sel.close()
        self.stop()
        raise TimeoutError("worker did not become ready in time")

    def kill(self) -> None:
        """Hard crash (SIGKILL), as a fault drill."""
        if self.proc and self.proc.poll() is None:
            self.proc.kill()
            self.proc.wait(timeout=10)
        if self.proc:
            LIVE.discard(self.proc.pid)

    def stop(self, timeout: float = 10.0) -> None:
        if self.proc is None:
            return
        if self.proc.poll() is None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=timeout)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.proc.wait(timeout=timeout)
        for f in (self.proc.stdout, self.proc.stderr):
            if f:
                f.close()
        LIVE.discard(self.proc.pid)

    @property
    def alive(self) -> bool:
        return self.proc is not None and self.proc.poll() is None


@dataclass
class LoopbackRing:
    preset: str = "tiny-llama-cpu"
    stages: int = 2
    seed: int = 0
    backend: str = "reference"
    topology: str = "loopback"
    model_revision: str = "random-seed"
    generation: int = 1
    procs: list[ManagedProcess] = field(default_factory=list)
    ports: list[int] = field(default_factory=list)
    layers: list[tuple[int, int]] = field(default_factory=list)

    def _args(self, i: int, next_port: int | None) -> list[str]:
        a = ["-m", "swarm_inference_lab_b200.runtime.worker", "--preset", self.preset,
             "--stage", str(i), "--stages", str(self.stages), "--seed", str(self.seed),
             "--generation", str(self.generation), "--topology", self.topology,
             "--model-revision", self.model_revision, "--backend", self.backend]
        if next_port is not None:
            a += ["--next", f"127.0.0.1:{next_port}"]
        return a

    def start(self) -> None:
        self.procs = [None] * self.stages  # type: ignore[list-item]
        self.ports = [0] * self.stages
        self.layers = [(0, 0)] * self.stages
        nxt = None
        for i in reversed(range(self.stages)):
            p = ManagedProcess(self._args(i, nxt))
            info = p.start()
            self.procs[i] = p
            self.ports[i] = info["port"]
            self.layers[i] = tuple(info["layers"])
            nxt = info["port"]

    def stop(self) -> None:
        for p in self.procs:
            if p is not None:
                p.stop()

    def route(self):
        from ..coordinator.session import Route
        return Route(stage0=("127.0.0.1", self.ports[0]), generation=self.generation,
                     topology_id=self.topology, model_revision=self.model_revision,
                     stage0_layers=self.layers[0])

    async def _install(self, i: int) -> None:
        conn = await StageRingConnection.open("127.0.0.1", self.ports[i], timeout=30)
        try:
            nxt = self.ports[i + 1] if i + 1 < self.stages else None
            msg = sr.StageMessage(
                operation=sr.Operation.LOAD_STAGE, model_revision=self.model_revision,
                tokenizer_revision="none", topology_id=self.topology, stage_id=i,
                layer_start=self.layers[i][0], layer_end=self.layers[i][1], session_id="",
                request_id="route", sequence_number=0, token_position=-1,
                source_stage=sr.COORDINATOR, destination_stage=i,
                attributes={"install_route": {
                    "generation": self.generation,
                    "next_hop": ["127.0.0.1", nxt] if nxt else None,
                    "next_layers": list(self.layers[i + 1]) if nxt else None}})
            rep = await conn.request(msg)
            if rep.operation == sr.Operation.ERROR:
                raise RuntimeError(f"route install failed on stage {i}: {rep.attributes}")
        finally:
            conn.close()

    async def recover(self, route, exc):
        """Restart dead workers, then install generation + 1 on every stage."""
        self.generation += 1
        for i in reversed(range(self.stages)):
            if not self.procs[i].alive:
                nxt = self.ports[i + 1] if i + 1 < self.stages else None
                p = ManagedProcess(self._args(i, nxt))
                info = p.start()
                self.procs[i] = p
                self.ports[i] = info["port"]
        for i in reversed(range(self.stages)):
            await self._install(i)
        return self.route()

    def __enter__(self):
        self.start()
        return self

    def __exit__(self, *exc):
        self.stop()


def run(coro):
    return asyncio.run(coro)
