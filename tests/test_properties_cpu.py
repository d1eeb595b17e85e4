"""Property tests (hypothesis) of the control plane's pure pieces: layer intervals cover the
model exactly once; replica placement uses distinct workers and its balancing never lowers
the weakest route; the route allocator never over-subscribes a route or a worker under any
interleaving of reserve / release / expiry; the durable generation never repeats."""
import pytest

hypothesis = pytest.importorskip("hypothesis")
from hypothesis import given, settings, strategies as st  # noqa: E402


@given(layers=st.integers(1, 200), stages=st.integers(1, 64))
def test_equal_layer_ranges_cover_every_layer_once(layers, stages):
    from swarm_inference_lab_b200.runtime.worker import equal_layer_ranges
    stages = min(stages, layers)
    r = equal_layer_ranges(layers, stages)
    assert len(r) == stages and r[0][0] == 0 and r[-1][1] == layers
    assert all(a[1] == b[0] for a, b in zip(r, r[1:]))
    sizes = [hi - lo for lo, hi in r]
    assert min(sizes) >= 1 and max(sizes) - min(sizes) <= 1


@given(speeds=st.lists(st.floats(1.0, 1000.0), min_size=2, max_size=24),
       replicas=st.integers(1, 4), stages=st.integers(1, 6))
def test_place_replicas_distinct_workers_and_balanced(speeds, replicas, stages):
    from swarm_inference_lab_b200.coordinator.replicas import place_replicas
    if replicas * stages > len(speeds):
        return
    ws = {f"w{i}": s for i, s in enumerate(speeds)}
    routes = place_replicas(ws, replicas, stages)
    used = [w for r in routes for w in r.workers]
    assert len(routes) == replicas and all(len(r.workers) == stages for r in routes)
    assert len(used) == len(set(used))
    # the fastest replicas * stages workers are the ones used
    fastest = sorted(ws.values(), reverse=True)[:replicas * stages]
    assert sorted((ws[w] for w in used), reverse=True) == fastest
    # every route's predicted step is its slowest stage
    for r in routes:
        assert r.step_ms == pytest.approx(1e3 / min(ws[w] for w in r.workers))


@settings(max_examples=60)
@given(ops=st.lists(st.tuples(st.sampled_from(["reserve", "release", "tick"]), st.integers(0, 3)),
                    max_size=80))
def test_route_allocator_never_over_subscribes(ops):
    from swarm_inference_lab_b200.coordinator.replicas import (AtomicRouteAllocator,
                                                               CapacityExhausted, ReplicaRoute)
    now = [0.0]
    routes = [ReplicaRoute(f"r{i}", [f"w{i}", "shared"], 2, 1.0) for i in range(3)]
    alloc = AtomicRouteAllocator(routes, ttl_s=5.0, clock=lambda: now[0])
    live = []
    for op, k in ops:
        if op == "reserve":
            rid = f"r{k % 3}"
            try:
                live.append(alloc.reserve(rid).lease_id)
            except CapacityExhausted:
                assert alloc.routes[rid].active == 2
        elif op == "release" and live:
            alloc.release(live.pop(k % len(live)))
        else:
            now[0] += 2.0                          # leases expire after 5 s
        alloc._reclaim()
        held = set(alloc.leases)
        for r in alloc.routes.values():
            assert 0 <= r.active <= r.capacity
        assert sum(r.active for r in alloc.routes.values()) == len(held)
        assert alloc.worker_load.get("shared", 0) == len(held)
        live = [l for l in live if l in held]


@settings(max_examples=25, deadline=None)
@given(steps=st.lists(st.integers(1, 5), min_size=1, max_size=6))
def test_generations_never_repeat_over_restarts(tmp_path_factory, steps):
    from swarm_inference_lab_b200.coordinator.deployment import DeploymentManager
    from swarm_inference_lab_b200.coordinator.state import DurableState, WorkerRegistry
    from swarm_inference_lab_b200.security.identity import Identity
    path = tmp_path_factory.mktemp("gen") / "state.json"
    ident = Identity.generate("c")
    seen = []
    for n in steps:                                # one coordinator life per entry
        dm = DeploymentManager(WorkerRegistry(), {}, ident, DurableState(path))
        seen += [dm._next_generation() for _ in range(n)]
    assert seen == sorted(seen) and len(seen) == len(set(seen))


_text = st.text(alphabet=st.characters(min_codepoint=33, max_codepoint=0x2FF), min_size=1, max_size=24)


@settings(max_examples=80, deadline=None)
@given(op=st.integers(1, 13), seq=st.integers(0, 2 ** 40), pos=st.integers(-1, 2 ** 31 - 1),
       src=st.integers(-1, 63), dst=st.integers(-1, 63), stage=st.integers(0, 63),
       lo=st.integers(0, 500), n=st.integers(1, 100), sid=_text, rid=_text, rev=_text,
       payload=st.binary(max_size=512),
       attrs=st.dictionaries(st.text(min_size=1, max_size=8),
                             st.one_of(st.integers(-10 ** 9, 10 ** 9), st.booleans(), st.text(max_size=8)),
                             max_size=4))
def test_stage_ring_frames_roundtrip_in_both_codecs(op, seq, pos, src, dst, stage, lo, n, sid, rid,
                                                    rev, payload, attrs):
    """Any valid frame survives encode -> decode unchanged, and the C++ codec writes the same
    bytes and reads back the same fields (when the native library is built)."""
    from swarm_inference_lab_b200.protocol import stage_ring as sr
    m = sr.StageMessage(operation=sr.Operation(op), model_revision=rev, tokenizer_revision="tok",
                        topology_id="topo", stage_id=stage, layer_start=lo, layer_end=lo + n,
                        session_id=sid, request_id=rid, sequence_number=seq, token_position=pos,
                        source_stage=src, destination_stage=dst, payload=payload, attributes=attrs)
    f = sr.encode(m)
    assert sr.decode(f) == m
    try:
        import torch  # noqa: F401 - the native library links against torch's runtime
        from swarm_inference_lab_b200 import _native
    except ImportError:
        return
    meta = sr.canonical_json(m.metadata())
    assert _native.ring_encode(op, 0, seq, pos, src, dst, meta, payload) == f
    assert _native.ring_decode(f) == (op, 0, seq, pos, src, dst, meta, payload)
