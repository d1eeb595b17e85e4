"""Node agent and runtime manager.

The runtime manager derives a node's runtime configuration: free TCP ports for
the control / data / probe services (bound and released to check availability),
the memory the stage owners may use (device memory minus a reserve, host memory
minus a reserve) and the endpoints to advertise.  The node agent is the
persistent per-node service: it owns the worker runtime (stage owners), the
network probe server and, on the coordinator node, the coordinator runtime; it
heartbeats the registry and restarts a crashed child with exponential backoff
(bounded attempts).

Reference: si/cluster/agent.py:78,167 (``NodeAgent``); si/cluster/runtime_manager.py:83.
"""
from __future__ import annotations

import socket
import time
from dataclasses import asdict, dataclass, field


def free_port(host: str = "127.0.0.1") -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind((host, 0))
        return s.getsockname()[1]


def port_available(port: int, host: str = "127.0.0.1") -> bool:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
        try:
            s.bind((host, port))
            return True
        except OSError:
            return False


@dataclass
class RuntimeConfig:
    host: str
    control_port: int
    data_port: int
    probe_port: int
    device_memory_bytes: list[int]
    host_memory_bytes: int
    advertise: dict = field(default_factory=dict)

    def to_json(self) -> dict:
        return asdict(self)


class RuntimeManager:
    def __init__(self, host: str = "127.0.0.1", *, device_reserve_frac: float = 0.05,
                 host_reserve_bytes: int = 8 << 30):
        self.host = host
        self.device_reserve = device_reserve_frac
        self.host_reserve = host_reserve_bytes

    def _pick(self, preferred: int | None) -> int:
        if preferred and port_available(preferred, self.host):
            return preferred
        return free_port(self.host)

    def configure(self, caps: dict, *, control: int | None = None, data: int | None = None,
                  probe: int | None = None) -> RuntimeConfig:
        ports = []
        for pref in (control, data, probe):
            p = self._pick(pref)
            while p in ports:
                p = free_port(self.host)
            ports.append(p)
        dev = [int(d["memory_gb"] * 1e9 * (1 - self.device_reserve)) for d in caps.get("devices", [])]
        hostb = max(0, int(caps.get("host_memory_gb", 0) * 1e9) - self.host_reserve)
        return RuntimeConfig(self.host, ports[0], ports[1], ports[2], dev, hostb,
                             {"control": f"{self.host}:{ports[0]}", "data": f"{self.host}:{ports[1]}",
                              "probe": f"{self.host}:{ports[2]}"})


@dataclass
class Child:
    name: str
    factory: object                      # () -> handle with .alive() and .stop()
    handle: object = None
    restarts: int = 0
    next_try: float = 0.0
    gave_up: bool = False


class NodeAgent:
    """Supervises the node's long-running children and heartbeats the registry."""

    def __init__(self, node_id: str, *, heartbeat=None, max_restarts: int = 5,
                 backoff_s: float = 1.0, backoff_max_s: float = 60.0, clock=time.monotonic):
        self.node_id = node_id
        self.heartbeat = heartbeat
        self.children: dict[str, Child] = {}
        self.max_restarts = max_restarts
        self.backoff, self.backoff_max = backoff_s, backoff_max_s
        self.clock = clock

    def add(self, name: str, factory) -> None:
        self.children[name] = Child(name, factory)

    def start(self) -> None:
        for c in self.children.values():
            if c.handle is None:
                c.handle = c.factory()

    def tick(self) -> dict:
        """One supervision round: heartbeat, restart dead children whose backoff elapsed."""
        now = self.clock()
        if self.heartbeat is not None:
            self.heartbeat(self.node_id)
        status = {}
        for c in self.children.values():
            if c.gave_up:
                status[c.name] = "failed"
                continue
            if c.handle is not None and c.handle.alive():
                status[c.name] = "running"
                continue
            if now < c.next_try:
                status[c.name] = "backoff"
                continue
            if c.restarts >= self.max_restarts:
                c.gave_up = True
                status[c.name] = "failed"
                continue
            c.restarts += 1
            c.next_try = now + min(self.backoff_max, self.backoff * 2 ** (c.restarts - 1))
            try:
                c.handle = c.factory()
                status[c.name] = "restarted"
            except Exception:  # noqa: BLE001 - counted as a failed attempt
                c.handle = None
                status[c.name] = "restart_failed"
        return status

    def stop(self) -> None:
        for c in reversed(list(self.children.values())):
            if c.handle is not None:
                try:
                    c.handle.stop()
                finally:
                    c.handle = None
