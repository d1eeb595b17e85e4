"""Replica data parallelism: atomic route reservations, replica placement, route scheduling.

* ``AtomicRouteAllocator``: each replica route has a capacity (concurrent sessions);
  ``reserve`` atomically claims a slot on every stage of a route (all or nothing),
  returns a lease with a TTL, ``release`` frees it, expired leases are reclaimed.
* ``place_replicas``: given workers with a measured per-stage throughput, builds
  ``replicas`` routes of ``stages`` workers each so that the slowest route is as
  fast as possible (greedy longest-processing-time assignment of the fastest
  workers to the weakest route, then balancing swaps).
* ``route_cost`` / ``ReplicaScheduler``: picks the route with the lowest predicted
  completion cost for a request (queue depth x step time + request tokens x step
  time, scaled by workload tier), among routes with free capacity.

Inside one box ``bench.py`` measures replica DP for the reference arm; this module
is the coordinator policy across replicas (GPU groups or hosts).

Reference: si/coordinator/reservations.py:90 ``AtomicRouteAllocator``;
si/coordinator/placement.py:77 ``place_replicas``; si/coordinator/scheduler.py:65,133.
"""
from __future__ import annotations

import itertools
import threading
import time
from dataclasses import dataclass, field


@dataclass
class ReplicaRoute:
    route_id: str
    workers: list[str]
    capacity: int
    step_ms: float                   # predicted decode step time of the route
    active: int = 0

    @property
    def free(self) -> int:
        return self.capacity - self.active


@dataclass
class RouteLeaseGrant:
    lease_id: str
    route_id: str
    expires_at: float


class CapacityExhausted(RuntimeError):
    pass


class AtomicRouteAllocator:
    def __init__(self, routes: list[ReplicaRoute], *, ttl_s: float = 300.0, clock=time.time):
        self.routes = {r.route_id: r for r in routes}
        self.ttl = ttl_s
        self.clock = clock
        self.leases: dict[str, RouteLeaseGrant] = {}
        self._lock = threading.Lock()
        self._ids = itertools.count()
        self.worker_load: dict[str, int] = {}

    def _reclaim(self) -> None:
        now = self.clock()
        for lid in [k for k, v in self.leases.items() if v.expires_at <= now]:
            self._free(lid)

    def _free(self, lease_id: str) -> None:
        g = self.leases.pop(lease_id, None)
        if g is None:
            return
        r = self.routes[g.route_id]
        r.active -= 1
        for w in r.workers:
            self.worker_load[w] -= 1

    def reserve(self, route_id: str) -> RouteLeaseGrant:
        with self._lock:
            self._reclaim()
            r = self.routes[route_id]
            if r.free <= 0:
                raise CapacityExhausted(f"route {route_id} is full")
            r.active += 1
            for w in r.workers:                       # every stage of the route, atomically
                self.worker_load[w] = self.worker_load.get(w, 0) + 1
            g = RouteLeaseGrant(f"L{next(self._ids)}", route_id, self.clock() + self.ttl)
            self.leases[g.lease_id] = g
            return g

    def add_route(self, route: ReplicaRoute) -> None:
        with self._lock:
            if route.route_id in self.routes:
                raise ValueError(f"route {route.route_id} exists")
            self.routes[route.route_id] = route

    def remove_route(self, route_id: str) -> None:
        """Removes an idle route (no live lease); a busy one raises ``CapacityExhausted``."""
        with self._lock:
            self._reclaim()
            r = self.routes[route_id]
            if r.active:
                raise CapacityExhausted(f"route {route_id} has {r.active} live lease(s)")
            del self.routes[route_id]

    def renew(self, lease_id: str) -> None:
        with self._lock:
            self.leases[lease_id].expires_at = self.clock() + self.ttl

    def release(self, lease_id: str) -> None:
        with self._lock:
            self._free(lease_id)


def place_replicas(worker_speed: dict[str, float], replicas: int, stages: int,
                   capacity: int = 8) -> list[ReplicaRoute]:
    """``worker_speed``: tokens/s one worker sustains for one stage of the model.  A route's
    step time is bounded by its slowest stage.  Returns ``replicas`` routes."""
    need = replicas * stages
    if len(worker_speed) < need:
        raise ValueError(f"need {need} workers, have {len(worker_speed)}")
    ws = sorted(worker_speed.items(), key=lambda kv: -kv[1])[:need]
    routes: list[list[tuple[str, float]]] = [[] for _ in range(replicas)]
    # Deal the fastest workers round-robin in a snake order so every route gets a similar mix.
    for i, w in enumerate(ws):
        rnd, pos = divmod(i, replicas)
        idx = pos if rnd % 2 == 0 else replicas - 1 - pos
        routes[idx].append(w)

    def bottleneck(r):
        return min(s for _, s in r)
    # Balancing swaps: raise the weakest route's bottleneck while it improves the minimum.
    improved = True
    while improved:
        improved = False
        order = sorted(range(replicas), key=lambda i: bottleneck(routes[i]))
        weak, strong = order[0], order[-1]
        wi = min(range(stages), key=lambda j: routes[weak][j][1])
        sj = max(range(stages), key=lambda j: routes[strong][j][1])
        a, b = routes[weak][wi], routes[strong][sj]
        if b[1] > a[1]:
            before = min(bottleneck(routes[weak]), bottleneck(routes[strong]))
            routes[weak][wi], routes[strong][sj] = b, a
            after = min(bottleneck(routes[weak]), bottleneck(routes[strong]))
            if after <= before:
                routes[weak][wi], routes[strong][sj] = a, b
            else:
                improved = True
    out = []
    for i, r in enumerate(routes):
        out.append(ReplicaRoute(f"replica{i}", [w for w, _ in r], capacity, 1e3 / bottleneck(r)))
    return out


TIER_WEIGHT = {"interactive": 1.0, "standard": 1.5, "batch": 3.0}


def route_cost(r: ReplicaRoute, prompt_tokens: int, output_tokens: int, tier: str = "standard") -> float:
    """Predicted milliseconds until the request completes on ``r`` (queueing included)."""
    queue = r.active * r.step_ms
    own = (output_tokens + prompt_tokens / 64.0) * r.step_ms * (1.0 + r.active / max(1, r.capacity))
    return (queue + own) / TIER_WEIGHT.get(tier, 1.0)


@dataclass
class ReplicaScheduler:
    allocator: AtomicRouteAllocator
    decisions: list = field(default_factory=list)

    def submit(self, prompt_tokens: int, output_tokens: int, tier: str = "standard") -> RouteLeaseGrant:
        cands = [r for r in self.allocator.routes.values() if r.free > 0]
        if not cands:
            raise CapacityExhausted("every replica route is full")
        best = min(cands, key=lambda r: (route_cost(r, prompt_tokens, output_tokens, tier), r.route_id))
        g = self.allocator.reserve(best.route_id)
        self.decisions.append((best.route_id, tier))
        return g
