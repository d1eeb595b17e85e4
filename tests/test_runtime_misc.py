"""Integrity audits, replay log, stage sessions, residency, engine processes, canonical facade (CPU)."""
import json
import sys

import pytest
import torch

from swarm_inference_lab_b200.coordinator.integrity import IntegrityCoordinator, ReputationBook
from swarm_inference_lab_b200.coordinator.replay_log import ReplayLog, ReplayLogError
from swarm_inference_lab_b200.runtime.processes import (EngineProcess, ProcessVerificationError, file_digest,
                                                        shutdown_all)
from swarm_inference_lab_b200.runtime.residency import ResidencyTracker
from swarm_inference_lab_b200.runtime.sessions import StageSessionRegistry


def test_integrity_quarantines_the_disagreeing_worker():
    ic = IntegrityCoordinator(ReputationBook(max_mismatches=2))
    a = torch.arange(10)
    assert ic.judge("w0", a, "w1", a.clone())
    for _ in range(2):
        assert not ic.judge("w2", a + 1, "w1", a, tiebreak=("w0", a.clone()))
    assert not ic.book.eligible("w2") and ic.book.eligible("w1")
    assert ic.judge("w0", torch.ones(3), "w1", torch.ones(3) + 1e-5, exact=False)


def test_replay_log_roundtrip_and_tamper_detection(tmp_path):
    log = ReplayLog(tmp_path)
    log.open("r1", [5, 6, 7])
    log.accept("r1", 3, 11)
    log.accept("r1", 4, 12)
    with pytest.raises(ReplayLogError):
        log.accept("r1", 9, 13)
    log.finish("r1")
    assert log.replay_inputs("r1") == [5, 6, 7, 11, 12]
    rec = ReplayLog(tmp_path).load("r1")
    assert rec.tokens == [11, 12] and rec.state == "finished"
    p = tmp_path / "r1.jsonl"
    p.write_text(p.read_text().replace("[3, 11]", "[3, 99]"))
    with pytest.raises(ReplayLogError, match="chain"):
        ReplayLog(tmp_path).load("r1")


def test_stage_sessions_generation_fence_ttl_and_lru():
    reg = StageSessionRegistry(max_sessions=2, idle_ttl_s=10)
    evicted = []
    reg.open("a", "t", 1, now=0)
    reg.open("b", "t", 1, now=1)
    reg.get("a", topology_id="t", generation=1, now=2)
    reg.open("c", "t", 2, now=3, evict=evicted.append)        # LRU evicts b
    assert [s.session_id for s in evicted] == ["b"]
    with pytest.raises(KeyError):
        reg.get("a", topology_id="t", generation=2)
    reg.advance("a", 5)
    with pytest.raises(ValueError):
        reg.advance("a", 4)
    assert reg.invalidate_generation(2) == ["a"]
    assert reg.expire(now=100) == ["c"]


def test_residency_tracker():
    rt = ResidencyTracker()
    rt.place("e0", "device:0", 100)
    rt.place("e1", "host_pinned", 50)
    rt.place("emb", "device:0", 10, pinned=True)
    assert rt.lookup("e0", "device:0") and not rt.lookup("e1", "device:0")
    rt.move("e1", "device:0", 0.001)
    assert rt.bytes_on() == {"device:0": 160}
    assert rt.moved_bytes(dst="device:0") == 50
    with pytest.raises(ValueError):
        rt.move("emb", "host")
    assert rt.evict_candidates("device:0", 60) == ["e0"]


def test_engine_process_verify_start_stop(tmp_path):
    script = tmp_path / "w.py"
    script.write_text("import json,time,sys\nprint(json.dumps({'ready': True, 'port': 1}), flush=True)\n"
                      "time.sleep(60)\n")
    p = EngineProcess([sys.executable, str(script)], verify={str(script): file_digest(script)})
    assert p.start(ready_timeout_s=30)["port"] == 1
    assert p.alive()
    assert shutdown_all([p], 10) == ["terminated"]
    bad = EngineProcess([sys.executable, str(script)], verify={str(script): "0" * 64})
    with pytest.raises(ProcessVerificationError):
        bad.start()


def test_canonical_runtime_dry_run():
    from swarm_inference_lab_b200.engines import ClusterCapabilities, RequestShape
    from swarm_inference_lab_b200.runtime.canonical import CanonicalRuntime
    rt = CanonicalRuntime()
    info = rt.inspect("kimi-k2-shape")
    assert info["mla"] and info["parameters"] > 9e11
    caps = ClusterCapabilities(nodes={"local": {"gpus": 8, "gpu_name": "NVIDIA B200"}})
    r = rt.dry_run("llama-3-8b-shape", caps, RequestShape(batch=32, prompt_tokens=2048,
                                                           output_tokens=256, mode="throughput"))
    assert r["winner"]["engine"] == "native-stage"
    json.dumps(r)


def test_network_probe_signed_ticket_and_repository():
    import asyncio

    from swarm_inference_lab_b200.cluster.network import (DirectedNetworkMeasurer, LinkRepository, ProbeServer,
                                                          issue_ticket)
    from swarm_inference_lab_b200.security.identity import Identity, SignatureError

    async def main():
        coord = Identity.generate("coord")
        srv = ProbeServer("w1", coord.fingerprint)
        port = await srv.start()
        t = issue_ticket(coord, "w0", "w1", nbytes=1 << 20)
        m = await DirectedNetworkMeasurer("w0", pings=5).measure("127.0.0.1", port, t)
        assert m.dst == "w1" and m.rtt_ms > 0 and m.upload_Bps > 0 and m.download_Bps > 0
        with pytest.raises(SignatureError):           # replayed ticket
            await DirectedNetworkMeasurer("w0", pings=2).measure("127.0.0.1", port, t)
        other = Identity.generate("rogue")
        with pytest.raises(SignatureError):           # untrusted signer
            await DirectedNetworkMeasurer("w0").measure("127.0.0.1", port, issue_ticket(other, "w0", "w1"))
        await srv.close()
        repo = LinkRepository(ttl_s=10)
        repo.record(m)
        assert repo.fresh("w0", "w1") is m
        assert repo.stale_links([("w0", "w1"), ("w1", "w0")]) == [("w1", "w0")]
        assert repo.fresh("w0", "w1", now=m.measured_at + 11) is None

    asyncio.run(main())


def test_tcp_meter_and_emulated_transport():
    import asyncio

    from swarm_inference_lab_b200.transport.emulated import EmulatedTransport, LinkDropped, LinkModel
    from swarm_inference_lab_b200.transport.tcp_meter import TcpMeterProxy

    async def main():
        async def echo(r, w):
            while True:
                b = await r.read(4096)
                if not b:
                    break
                w.write(b)
                await w.drain()
            w.close()
        up = await asyncio.start_server(echo, "127.0.0.1", 0)
        proxy = TcpMeterProxy("127.0.0.1", up.sockets[0].getsockname()[1])
        port = await proxy.start()
        r, w = await asyncio.open_connection("127.0.0.1", port)
        w.write(b"x" * 10000)
        await w.drain()
        got = b""
        while len(got) < 10000:
            got += await r.read(4096)
        w.close()
        await asyncio.sleep(0.05)
        assert proxy.stats.bytes_up == 10000 and proxy.stats.bytes_down == 10000
        await proxy.close()
        up.close()

        async def handler(msg):
            return [msg]
        from swarm_inference_lab_b200.protocol import stage_ring as sr
        msg = sr.StageMessage(operation=sr.Operation.HEALTH, model_revision="m", tokenizer_revision="t",
                              topology_id="x", stage_id=0, layer_start=0, layer_end=1, session_id="s",
                              request_id="r", sequence_number=0, token_position=0, source_stage=0,
                              destination_stage=0)
        em = EmulatedTransport(handler, LinkModel(latency_s=1e-3, bandwidth_Bps=1e6))
        await em.request(msg)
        t1 = em.clock.now
        assert t1 > 2e-3
        em2 = EmulatedTransport(handler, LinkModel(latency_s=1e-3, bandwidth_Bps=1e6))
        await em2.request(msg)
        assert em2.clock.now == t1                      # deterministic
        drop = EmulatedTransport(handler, LinkModel(drop_prob=1.0))
        with pytest.raises(LinkDropped):
            await drop.request(msg)

    asyncio.run(main())


def test_simulation_ring_and_expert_layer():
    from swarm_inference_lab_b200.testing.simulation import (Link, StageNode, expert_layer_time, simulate_ring,
                                                             zipf_tokens)

    def ring(churn=(), corruption=0.0):
        stages = [StageNode("s0", 0.010, 1e-4), StageNode("s1", 0.020, 1e-4)]
        return simulate_ring(stages, Link(latency_s=1e-3, bandwidth_Bps=1e9, corruption=corruption),
                             requests=4, prompt_tokens=32, output_tokens=16, hidden_bytes=8192,
                             churn=churn, seed=1)
    a, b = ring(), ring()
    assert a == b and a["completed"] == 4                      # deterministic
    # four requests share the 20 ms bottleneck stage: ~50 tokens/s, TPOT ~ 4 x 20 ms
    assert 0.07 < a["tpot_p50_s"] < 0.09
    assert 40 < a["tokens_per_s"] < 55
    c = ring(churn=[(0.2, 1, 0.5)])
    assert c["completed"] == 4 and c["replays"] > 0 and c["sim_time_s"] > a["sim_time_s"]
    d = ring(corruption=0.3)
    assert d["resends"] > 0
    even = expert_layer_time([10] * 8, [i // 2 for i in range(8)], 4, flops_per_token=1e9, rate_flops=1e15,
                             weight_bytes_per_expert=4e7, hbm_Bps=6e12, token_bytes=14336, link_Bps=7e11,
                             link_latency_s=1e-5)
    skew = zipf_tokens(8, 64, 2, skew=1.5)
    uneven = expert_layer_time(skew, [i // 2 for i in range(8)], 4, flops_per_token=1e9, rate_flops=1e15,
                               weight_bytes_per_expert=4e7, hbm_Bps=6e12, token_bytes=14336,
                               link_Bps=7e11, link_latency_s=1e-5)
    assert even["imbalance"] == pytest.approx(1.0) and uneven["imbalance"] > 1.0


def test_coordinator_runtime_partial_start_rollback():
    import asyncio

    from swarm_inference_lab_b200.coordinator.runtime import CoordinatorRuntime
    log = []
    rt = CoordinatorRuntime()
    rt.add("state", lambda: log.append("start state"), lambda: log.append("stop state"))

    async def boom():
        raise RuntimeError("port in use")
    rt.add("server", boom, lambda: log.append("stop server"))
    with pytest.raises(RuntimeError):
        asyncio.run(rt.start())
    assert log == ["start state", "stop state"] and not rt.running
    ok = CoordinatorRuntime()
    ok.add("a", lambda: log.append("a"), lambda: log.append("-a"))
    asyncio.run(ok.start())
    asyncio.run(ok.start())                      # idempotent
    asyncio.run(ok.stop())
    assert log[-2:] == ["a", "-a"]


def test_model_catalog_and_node_agent():
    from swarm_inference_lab_b200.cluster.agent import NodeAgent, RuntimeManager
    from swarm_inference_lab_b200.coordinator.catalog import ModelCatalog, ModelReport, probe_report
    cat = ModelCatalog()
    cat.report(probe_report("w0", "llama-3-8b-shape"))
    cat.report(ModelReport("w1", "m", "rev-a", "qwen3", 10, 2, True, reported_at=1))
    cat.report(ModelReport("w2", "m", "rev-a", "qwen3", 10, 2, True, reported_at=2))
    cat.report(ModelReport("w3", "m", "rev-b", "qwen3", 10, 2, True, reported_at=3))
    assert cat.resolve("m").revision == "rev-a" and cat.holders("rev-a") == ["w1", "w2"]
    assert cat.resolve("llama-3-8b-shape").family == "llama"
    cat.forget_worker("w1")
    assert cat.holders("rev-a") == ["w2"]
    cfg = RuntimeManager().configure({"devices": [{"memory_gb": 180}], "host_memory_gb": 64})
    assert len({cfg.control_port, cfg.data_port, cfg.probe_port}) == 3
    assert cfg.device_memory_bytes[0] < 180e9

    class H:
        def __init__(self):
            self.up = True

        def alive(self):
            return self.up

        def stop(self):
            self.up = False
    t = [0.0]
    made = []

    def factory():
        h = H()
        made.append(h)
        return h
    beats = []
    ag = NodeAgent("n0", heartbeat=beats.append, max_restarts=2, backoff_s=1.0, clock=lambda: t[0])
    ag.add("worker", factory)
    ag.start()
    assert ag.tick() == {"worker": "running"}
    made[-1].up = False
    assert ag.tick() == {"worker": "restarted"}
    made[-1].up = False
    assert ag.tick() == {"worker": "backoff"}
    t[0] = 5.0
    assert ag.tick() == {"worker": "restarted"}
    made[-1].up = False
    t[0] = 100.0
    assert ag.tick() == {"worker": "failed"}
    assert len(beats) == 5
    ag.stop()


def test_compatibility_registry_and_engine_leases(tmp_path):
    from swarm_inference_lab_b200.engines.compat import CompatibilityRegistry, engine_facts, probe_native_stage
    from swarm_inference_lab_b200.engines.worker_control import EngineController, issue_engine_lease
    from swarm_inference_lab_b200.security.identity import Identity, SignatureError
    facts = engine_facts({"devices": [{"capability": "10.0", "memory_gb": 183}], "host_memory_gb": 2000})
    assert facts["sm100a_kernels"] and "fp8_e4m3" in facts["dtypes"]
    reg = CompatibilityRegistry(tmp_path / "compat.json")
    assert probe_native_stage(reg, facts, "llama", "bf16", lambda: None).ok

    def bad():
        raise RuntimeError("kernel failed")
    assert not probe_native_stage(reg, facts, "deepseek_v3", "fp8_block128", bad).ok
    again = CompatibilityRegistry(tmp_path / "compat.json")
    assert again.check("native-stage", "deepseek_v3", "fp8_block128", "b200")[0] is False
    assert again.check("native-stage", "qwen3", "bf16", "b200") == (True, "unprobed", 0.9)
    cpu = engine_facts({"devices": []})
    assert not probe_native_stage(reg, cpu, "llama", "bf16", lambda: None).ok

    coord, worker = Identity.generate("c"), Identity.generate("w")
    t = [1000.0]
    started = []

    class Handle:
        def __init__(self, n):
            self.n = n
            started.append(n)

        def stop(self):
            started.remove(self.n)
    ctl = EngineController(worker.fingerprint, coord.fingerprint, lambda e, rev: Handle(e), clock=lambda: t[0])
    lease = issue_engine_lease(coord, worker_fingerprint=worker.fingerprint, engine="native-stage",
                               model_revision="r1", generation=1, ttl_s=60)
    assert ctl.apply(lease) == "started" and started == ["native-stage"]
    with pytest.raises(SignatureError):
        ctl.apply(lease)                              # replay
    other = issue_engine_lease(coord, worker_fingerprint="someone-else", engine="x", model_revision="r",
                               generation=2)
    with pytest.raises(SignatureError):
        ctl.apply(other)
    t[0] = 1e12
    assert ctl.sweep() == ["native-stage"] and started == []


def test_tensor_paths_and_shard_manager(tmp_path):
    from swarm_inference_lab_b200.model_io.resolver import ModelSourceResolver
    from swarm_inference_lab_b200.runtime.shard_manager import ShardIntegrityError, ShardLimitError, ShardManager
    from swarm_inference_lab_b200.transport.tensor_paths import choose_path
    t = torch.randn(3, 5)
    for same_proc, same_host in ((True, True), (False, True), (False, False)):
        p = choose_path(same_proc, same_host, peer_access=False)
        assert torch.equal(p.recv(p.send(t)), t), p.name
    import importlib.util
    import pathlib
    spec = importlib.util.spec_from_file_location("tmio", pathlib.Path(__file__).with_name("test_model_io.py"))
    tmio = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(tmio)
    _tiny_ckpt = tmio._tiny_ckpt
    ck = tmp_path / "ck"
    ck.mkdir()
    _tiny_ckpt(ck)
    res = ModelSourceResolver().inspect(str(ck))
    sm = ShardManager(budget_bytes=res.stage_bytes(0, 1, embed=True, head=False))
    st = sm.load_stage(res, 0, 1, embed=True, head=False)
    assert "model.embed_tokens.weight" in st.tensors and all(".layers.1." not in n for n in st.tensors)
    with pytest.raises(ShardLimitError):
        sm.load_stage(res, 1, 2, embed=False, head=True)
    sm.unload(st.key)
    assert sm.used == 0
    with pytest.raises(ShardIntegrityError):
        ShardManager(budget_bytes=1 << 30).load_stage(res, 1, 2, embed=False, head=True,
                                                      file_digests={"x": "0"})


def test_grpc_control_envelopes_and_chunk_stream():
    import asyncio

    from swarm_inference_lab_b200.transport.grpc_control import (EnvelopeError, GrpcControlClient,
                                                                 GrpcControlServer, pack, unpack)
    k, o = unpack(pack("WorkerHello", {"b": 1, "a": [1, 2]}))
    assert k == "WorkerHello" and o == {"a": [1, 2], "b": 1}
    assert pack("X", {"b": 1, "a": 2}).value == b'{"a":2,"b":1}'

    async def main():
        workers = {}

        async def register(kind, obj):
            workers[obj["worker_id"]] = obj
            return "RegisterAck", {"accepted": True, "count": len(workers)}

        async def echo_stream(tid, data):
            return data[::-1]
        srv = GrpcControlServer({("swarm.v1.Coordinator", "Register"): register},
                                stream_handler=echo_stream)
        port = await srv.start()
        cli = GrpcControlClient(f"127.0.0.1:{port}")
        kind, rep = await cli.call("swarm.v1.Coordinator", "Register", "WorkerRegistration",
                                   {"worker_id": "w0", "gpus": 8}, expect="RegisterAck")
        assert rep == {"accepted": True, "count": 1}
        data = bytes(range(256)) * 12000           # ~3 MB, several chunks
        out = await cli.execute_stream("t0", data, chunk_bytes=1 << 20)
        assert out == data[::-1]
        with pytest.raises(EnvelopeError):
            await cli.call("swarm.v1.Coordinator", "Register", "WorkerRegistration", {"worker_id": "w1"},
                           expect="Other")
        await cli.close()
        await srv.stop()

    asyncio.run(main())


def test_replica_placement_reservations_and_scheduler():
    from swarm_inference_lab_b200.coordinator.replicas import (AtomicRouteAllocator, CapacityExhausted,
                                                               ReplicaScheduler, place_replicas)
    speeds = {f"w{i}": s for i, s in enumerate([100, 90, 80, 70, 60, 50])}
    routes = place_replicas(speeds, replicas=2, stages=3, capacity=2)
    bott = sorted(min(speeds[w] for w in r.workers) for r in routes)
    assert len(routes) == 2 and all(len(r.workers) == 3 for r in routes)
    assert bott[0] >= 50 and len({w for r in routes for w in r.workers}) == 6
    t = [0.0]
    alloc = AtomicRouteAllocator(routes, ttl_s=10, clock=lambda: t[0])
    sch = ReplicaScheduler(alloc)
    grants = [sch.submit(100, 50) for _ in range(4)]
    assert {g.route_id for g in grants} == {"replica0", "replica1"}
    with pytest.raises(CapacityExhausted):
        sch.submit(100, 50)
    alloc.release(grants[0].lease_id)
    sch.submit(100, 50)
    t[0] = 100.0                                     # every lease expired -> reclaimed
    alloc.reserve("replica0")
    assert alloc.routes["replica0"].active == 1 and alloc.routes["replica1"].active == 0
    assert all(v in (0, 1) for v in alloc.worker_load.values())


def test_platform_adapters_and_acceptance(tmp_path):
    from swarm_inference_lab_b200 import platforms
    from swarm_inference_lab_b200.testing.acceptance import model_matrix, pre_physical_gate, write_evidence
    lx = platforms.LinuxAdapter()
    unit = lx.service_definition(["/usr/bin/python3", "-m", "swarm_inference_lab_b200.cli", "node", "run"])
    assert "ExecStart=/usr/bin/python3 -m" in unit and "Restart=on-failure" in unit
    assert "tcp dport { 7000, 7001 }" in lx.firewall_rules([7001, 7000])
    assert "host_memory_gb" in lx.hardware()
    assert "<key>Label</key>" in platforms.MacAdapter().service_definition(["a"])
    assert platforms.WindowsAdapter().service_definition(["C:\\\\x.exe"]).startswith("sc.exe create")
    gate = pre_physical_gate()
    assert gate["ok"], gate
    rows = {r["model"]: r for r in model_matrix()}
    assert rows["llama-3-8b-shape"]["fits"] and rows["kimi-k2-shape"]["params"] > 9e11
    p = write_evidence(gate, tmp_path)
    assert p.exists()


def test_synthetic_stages_are_deterministic_and_calibrated():
    import time as _t

    from swarm_inference_lab_b200.runtime.executors import StageSpec
    from swarm_inference_lab_b200.runtime.synthetic import SyntheticStageExecutor, calibrate

    def ring(seed):
        s0 = SyntheticStageExecutor(StageSpec(0, 0, 2, 2), 16, 1000, seed=seed)
        s1 = SyntheticStageExecutor(StageSpec(1, 2, 4, 2), 16, 1000, seed=seed,
                                    calib=calibrate(2.0, 0.0))
        for s in (s0, s1):
            s.open("a")
        toks, pos, cur = [], 0, torch.tensor([1, 2, 3])
        for _ in range(4):
            t = s1.forward("a", s0.forward("a", cur, pos), pos)
            pos += cur.shape[0]
            cur = t[-1:]
            toks.append(int(cur))
        return toks
    t0 = _t.perf_counter()
    a = ring(0)
    assert _t.perf_counter() - t0 >= 0.006          # three decode steps x 2 ms on stage 1
    assert a == ring(0) and a != ring(1)


def test_universal_worker_abi_and_queue():
    import asyncio

    from swarm_inference_lab_b200.runtime.abi import ExecutionQueue, GreedyVerifier, UniversalWorker

    class Backend:
        def __init__(self):
            self.batched = 0

        @staticmethod
        def next_token(ctx):
            return (sum(ctx) * 7 + len(ctx)) % 50

        def generate(self, prompt, max_new_tokens):
            out, ctx = [], list(prompt)
            for _ in range(max_new_tokens):
                t = self.next_token(ctx)
                out.append(t)
                ctx.append(t)
            return {"tokens": out}

        def generate_batch(self, jobs):
            self.batched += len(jobs)
            return [self.generate(**j) for j in jobs]

        def verify(self, context, candidates):
            return GreedyVerifier(self.next_token).verify(context, candidates)

    be = Backend()
    w = UniversalWorker(be)
    gen = w.run({"kind": "generate", "prompt": [1, 2], "max_new_tokens": 4, "job_id": "a"})
    assert gen["status"] == "OK" and len(gen["result"]["tokens"]) == 4
    toks = gen["result"]["tokens"]
    ok = w.run({"kind": "verify", "context": [1, 2], "candidates": toks[:3] + [toks[3] + 1]})
    assert ok["result"] == {"accepted": 3, "next": toks[3]}
    assert w.run({"kind": "draft", "context": [1], "k": 2})["status"] == "REJECTED"
    assert w.run({"kind": "nope"})["status"] == "REJECTED"

    async def main():
        q = ExecutionQueue(w, max_pending=16, max_batch=8)
        await q.start()
        res = await asyncio.gather(*[q.submit({"kind": "generate", "prompt": [i], "max_new_tokens": 2,
                                               "job_id": i}) for i in range(6)])
        await q.close()
        return res
    res = asyncio.run(main())
    assert all(r["status"] == "OK" for r in res) and [r["job_id"] for r in res] == list(range(6))
    assert be.batched >= 2


def test_decode_split_heuristics():
    from swarm_inference_lab_b200.ops import attention, mla
    assert attention.decode_splits(32, 8, 34) == 1          # 256 CTAs: one wave, nothing to merge
    assert attention.decode_splits(64, 8, 34) == 1
    assert attention.decode_splits(32, 1, 34) == 8          # one rank of TP8
    assert attention.decode_splits(32, 4, 34) == 2
    assert attention.decode_splits(1, 8, 34) == 8           # at most 8 splits
    assert attention.decode_splits(1, 8, 6) == 3            # never below 2 pages per split
    assert attention.decode_splits(128, 8, 1) == 1
    assert mla.decode_splits(32, 4096) == 4 and mla.decode_splits(1, 4096) == 64


def test_shipped_configs_validate():
    """Every shipped network profile validates as a NetworkProfile (and classifies into the
    expected topology domain), every node profile as a NodeProfile, the product config (with
    its relative includes) as a ProductConfig, and the WAN harness uses the profiles' RTTs."""
    from pathlib import Path

    from swarm_inference_lab_b200.config import NetworkProfile, NodeProfile, ProductConfig, load_yaml
    from swarm_inference_lab_b200.planner.topology import LinkProfile, classify
    from swarm_inference_lab_b200.testing.wan_ring import PROFILES
    root = Path(__file__).resolve().parents[1] / "configs"
    nets = {p.stem: NetworkProfile.from_yaml(p) for p in (root / "networks").glob("*.yaml")}
    assert {"nvlink5", "loopback", "wifi", "regional-wan", "global-wan"} <= set(nets)
    dom = {k: classify(LinkProfile("a", "b", v.rtt_ms, v.bandwidth_mbps / 8, jitter_ms=v.jitter_ms,
                                   stability=v.stability)).value for k, v in nets.items()}
    assert dom["regional-wan"] == "regional" and dom["global-wan"] == "wan"
    for p in (root / "nodes").glob("*.yaml"):
        NodeProfile(**load_yaml(p))
    for p in (root / "product").glob("b200-*.yaml"):
        assert ProductConfig.from_yaml(p).max_recoveries == 3
    assert PROFILES["global"] == nets["global-wan"].rtt_ms / 2e3


def test_cost_model_modes_and_unmeasured_penalty():
    """Serial token path and bottleneck-bound aggregate; each unmeasured input costs 2% of the
    score; the modes rank a fast-TTFT plan and a high-throughput plan differently."""
    import math

    from swarm_inference_lab_b200.planner.cost_model import PlanCostInputs, score_costs
    c = PlanCostInputs(stage_compute_ms=[4.0, 6.0], boundary_ms=[1.0], prefill_ms=100.0, batch=8)
    r = score_costs(c, "throughput")
    assert r.tpot_ms == 11.0 and r.bottleneck_ms == 6.0 and r.ttft_ms == 101.0
    assert math.isclose(r.decode_tok_s, 1000 / 11)
    assert math.isclose(r.aggregate_tok_s, 8 * 1000 / max(6.0 * 2, 11.0))
    pen = score_costs(PlanCostInputs([4.0, 6.0], [1.0], 100.0, batch=8, unmeasured=["a", "b"]),
                      "throughput")
    assert math.isclose(pen.score, r.score * 0.98 ** 2)
    fast = PlanCostInputs([5.0], [], prefill_ms=50.0, batch=1)        # one stage, low latency
    wide = PlanCostInputs([3.0] * 4, [0.5] * 3, prefill_ms=400.0, batch=32, replicas=2)
    assert score_costs(fast, "speed").score > score_costs(wide, "speed").score
    assert score_costs(wide, "throughput").score > score_costs(fast, "throughput").score
    roomy = PlanCostInputs([5.0], [], 50.0, memory_fraction=0.2)
    full = PlanCostInputs([5.0], [], 50.0, memory_fraction=0.9)
    assert score_costs(roomy, "capacity").score > score_costs(full, "capacity").score


def test_host_capabilities_and_doctor_report():
    from swarm_inference_lab_b200.doctor import run_doctor
    from swarm_inference_lab_b200.worker_caps import local_capabilities
    caps = local_capabilities(benchmark=False)
    assert caps["cpus"] and caps["os"] and caps["gpus"] == len(caps["devices"])
    rep = run_doctor()
    assert "checks" in rep and "torch" in rep["checks"] and "ok" in rep
    assert rep["checks"]["kernel_library"] in ("built",) or rep["checks"]["kernel_library"].startswith("missing")


def test_torch_rank_backend_serves_the_worker_abi_exactly():
    """The exact PyTorch backend behind ``UniversalWorker``: generate equals the reference
    greedy decode; verify accepts the greedy continuation whole and a corrupted draft up to its
    first wrong token (the same as the one-call-per-token ``GreedyVerifier``); draft proposes
    from the context; an integrity audit finds a tampered continuation."""
    from swarm_inference_lab_b200.models.config import TINY_LLAMA_CPU
    from swarm_inference_lab_b200.models.reference import ReferenceDecoder, random_source
    from swarm_inference_lab_b200.runtime.abi import GreedyVerifier, UniversalWorker
    from swarm_inference_lab_b200.runtime.torch_rank import TorchRankBackend
    torch.set_num_threads(2)
    prompt = [5, 9, 14, 5, 9, 22, 31]
    expect = ReferenceDecoder(TINY_LLAMA_CPU, random_source(0)).greedy_generate(prompt, 6)[0]
    be = TorchRankBackend({"preset": "tiny-llama-cpu", "seed": 0})
    w = UniversalWorker(be, "torch-rank")
    r = w.run({"kind": "generate", "prompt": prompt, "max_new_tokens": 6})
    assert r["status"] == "OK" and r["result"]["tokens"] == expect
    r = w.run({"kind": "verify", "context": prompt, "candidates": expect[:4]})
    assert r["result"] == {"accepted": 4, "next": expect[4]}
    bad = expect[:2] + [(expect[2] + 1) % 32000, expect[3]]
    r = w.run({"kind": "verify", "context": prompt, "candidates": bad})
    gv = GreedyVerifier(lambda ctx: be.generate(ctx, 1)["tokens"][0])
    assert r["result"] == gv.verify(prompt, bad) == {"accepted": 2, "next": expect[2]}
    # the trailing bigram (5, 9) last occurred at positions 3-4, followed by 22, 31, 5
    r = w.run({"kind": "draft", "context": prompt + [5, 9], "k": 3})
    assert r["result"]["draft"] == [22, 31, 5]
    tampered = expect[:3] + [expect[3] + 1] + expect[4:]
    r = w.run({"kind": "background", "name": "integrity_audit",
               "args": {"prompt": prompt, "tokens": tampered}})
    assert r["result"]["agreed"] is False and r["result"]["first_mismatch"] == 3
    r = w.run({"kind": "background", "name": "integrity_audit",
               "args": {"prompt": prompt, "tokens": expect}})
    assert r["result"]["agreed"] is True
