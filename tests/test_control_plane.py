"""Control plane on CPU: identities, leases, TLS, pairing, state, planner, engines, CLI."""
import asyncio
import json
import time

import pytest

from swarm_inference_lab_b200.security.identity import (Identity, LeaseVerifier, RouteLease,
                                                        SignatureError, StageAssignment, issue_lease,
                                                        sign_record, verify_record)


def _lease(gen=1, ttl=60.0, wfp="sha256:w"):
    return RouteLease("topo", gen, "rev", "tok", "dense", "bfloat16",
                      [StageAssignment(0, "w0", wfp, 0, 2, "127.0.0.1:1", "127.0.0.1:2")],
                      expires_at=time.time() + ttl)


def test_signatures_and_tamper():
    a = Identity.generate("a")
    rec = sign_record(a, {"x": 1})
    assert verify_record(rec, {a.fingerprint})["x"] == 1
    rec2 = dict(rec, x=2)
    with pytest.raises(SignatureError):
        verify_record(rec2)
    with pytest.raises(SignatureError):
        verify_record(rec, {"sha256:someone-else"})


def test_identity_persistence(tmp_path):
    p = tmp_path / "id.json"
    a = Identity.load_or_create(p, "n")
    b = Identity.load(p)
    assert a.fingerprint == b.fingerprint
    assert (p.stat().st_mode & 0o777) == 0o600


def test_route_lease_rules():
    coord = Identity.generate("coord")
    v = LeaseVerifier(coord.fingerprint)
    signed = issue_lease(coord, _lease(gen=1))
    v.verify(signed, worker_fingerprint="sha256:w", model_revision="rev")
    with pytest.raises(SignatureError, match="nonce|stale"):
        v.verify(signed)  # replay
    with pytest.raises(SignatureError, match="stale"):
        v.verify(issue_lease(coord, _lease(gen=1)))
    with pytest.raises(SignatureError, match="expired"):
        v.verify(issue_lease(coord, _lease(gen=5, ttl=-1)))
    other = Identity.generate("evil")
    with pytest.raises(SignatureError, match="untrusted"):
        v.verify(issue_lease(other, _lease(gen=9)))
    with pytest.raises(SignatureError, match="does not assign"):
        v.verify(issue_lease(coord, _lease(gen=10)), worker_fingerprint="sha256:other")


def test_tls_cert_binds_fingerprint():
    from swarm_inference_lab_b200.security.tls import cert_fingerprint_binding, create_ca, issue_node_cert
    ca = create_ca("c")
    node = issue_node_cert(ca, "n1", "sha256:abc", ["127.0.0.1", "node1"])
    assert cert_fingerprint_binding(node.cert) == "sha256:abc"


def test_pairing_end_to_end(tmp_path):
    from swarm_inference_lab_b200.cluster.pairing import PairingError, PairingManager, join
    from swarm_inference_lab_b200.cluster.state import ClusterStateStore
    from swarm_inference_lab_b200.security.tls import cert_fingerprint_binding, create_ca
    coord = ClusterStateStore(tmp_path / "coord")
    ca = create_ca("lab")

    async def go():
        pm = PairingManager(coord, "127.0.0.1:0")
        port = await pm.start("127.0.0.1", 0)
        pm.endpoint = f"127.0.0.1:{port}"
        coord.create_cluster("lab", pm.endpoint, ca.cert, ca.key)
        inv = pm.invite()
        node = ClusterStateStore(tmp_path / "node")
        rep = await join(inv.uri(), node, "gpu-node-1", capabilities={"gpus": 8})
        # single use
        with pytest.raises(PairingError):
            await join(inv.uri(), ClusterStateStore(tmp_path / "node2"), "n2")
        await pm.close()
        return node, rep
    node, rep = asyncio.run(go())
    assert rep["cluster"] == "lab"
    members = coord.load_cluster()["members"]
    assert "gpu-node-1" in members and members["gpu-node-1"]["capabilities"]["gpus"] == 8
    cert = (node.root / "tls" / "node.crt").read_bytes()
    assert cert_fingerprint_binding(cert) == node.identity().fingerprint
    fp = coord.revoke("gpu-node-1")
    assert fp in coord.load_cluster()["revoked"]


def test_durable_state_and_restart(tmp_path):
    from swarm_inference_lab_b200.coordinator.state import DurableState
    s = DurableState(tmp_path / "s.json")
    s.record_request("r1", [1, 2], {"max_new_tokens": 4})
    s.accept_token("r1", 7)
    s2 = DurableState(tmp_path / "s.json")
    assert s2.replay_tokens("r1") == [1, 2, 7]
    assert s2.mark_restart_boundaries() == ["r1"]
    assert s2.data["requests"]["r1"]["state"] == "replay_required"


def test_event_stream_order():
    from swarm_inference_lab_b200.coordinator.state import EventStream

    async def go():
        es = EventStream("r")
        for i in range(3):
            await es.put("TOKEN_GENERATED", token=i)
        await es.put("REQUEST_COMPLETED")
        return [e async for e in es]
    evs = asyncio.run(go())
    assert [e["seq"] for e in evs] == [1, 2, 3, 4]


def test_registry_heartbeats():
    from swarm_inference_lab_b200.coordinator.state import WorkerRecord, WorkerRegistry
    r = WorkerRegistry(heartbeat_timeout_s=10)
    r.register(WorkerRecord("w1", "fp", "e"))
    r.workers["w1"].last_heartbeat -= 20
    assert r.sweep() == ["w1"] and not r.healthy()


def test_trace_critical_path(tmp_path):
    from swarm_inference_lab_b200.telemetry.trace import TraceWriter, critical_path, read_trace
    tw = TraceWriter(tmp_path / "t.jsonl", "p")
    with tw.span("prefill") as a:
        time.sleep(0.01)
    with tw.span("recv_token", after=[a]):
        time.sleep(0.005)
    tw.close()
    cp = critical_path(read_trace(tmp_path / "t.jsonl"))
    assert cp["path"] == ["prefill", "recv_token"] and cp["token_critical_receives"] == 1


def test_chrome_trace_export(tmp_path):
    """Two processes' JSONL traces merge into one Chrome trace: complete events in
    microseconds, instant events, process names and a flow arrow for the causal link."""
    import json as _json

    from swarm_inference_lab_b200.telemetry.trace import TraceWriter, write_chrome_trace
    a = TraceWriter(tmp_path / "a.jsonl", "stage0")
    b = TraceWriter(tmp_path / "b.jsonl", "stage1")
    with a.span("forward", layers=16) as sa:
        time.sleep(0.002)
    with b.span("recv_activation", after=[sa]):
        time.sleep(0.001)
    b.event("token", index=0)
    a.close()
    b.close()
    out = write_chrome_trace([tmp_path / "a.jsonl", tmp_path / "b.jsonl"], tmp_path / "t.json")
    ev = _json.loads(out.read_text())["traceEvents"]
    names = {e["args"]["name"] for e in ev if e["ph"] == "M"}
    assert names == {"stage0", "stage1"}
    fwd = next(e for e in ev if e["ph"] == "X" and e["name"] == "forward")
    rcv = next(e for e in ev if e["ph"] == "X" and e["name"] == "recv_activation")
    assert fwd["dur"] >= 2000 and fwd["args"]["layers"] == 16 and rcv["ts"] >= fwd["ts"] + fwd["dur"]
    assert any(e["ph"] == "i" and e["name"] == "token" for e in ev)
    s_, f_ = [e for e in ev if e["ph"] == "s"], [e for e in ev if e["ph"] == "f"]
    assert len(s_) == len(f_) == 1 and s_[0]["pid"] != f_[0]["pid"]


def test_box_planner_refit_changes_choice():
    from swarm_inference_lab_b200.models.config import LLAMA3_8B
    from swarm_inference_lab_b200.planner.box_planner import BoxMeasurements, plan_box
    fast = BoxMeasurements(ar_alpha_us=2.0, ar_beta_us_per_mb=1.0)
    slow = BoxMeasurements(ar_alpha_us=400.0, ar_beta_us_per_mb=50.0)
    pf = plan_box(LLAMA3_8B, 8, fast, batch=32, ctx=2304, prompt=2048)[0]
    ps = plan_box(LLAMA3_8B, 8, slow, batch=32, ctx=2304, prompt=2048)[0]
    assert pf.tp == 8          # cheap all-reduce: tensor parallel everywhere
    assert ps.tp < 8           # expensive all-reduce: the refit planner backs off TP
    m = BoxMeasurements()
    m.fit_allreduce([(8192, 10.0), (1 << 20, 12.6), (4 << 20, 20.4)])
    assert abs(m.ar_beta_us_per_mb - 2.6) < 0.2 and "ar_alpha_us" in m.measured
    m.fit_decode([(20e9, 260, 6.29), (10e9, 260, 4.0), (2e9, 260, 2.0)])
    assert 0 < m.eta <= 1 and m.launch_us >= 0


def test_stage_planner_prefers_fast_links():
    from swarm_inference_lab_b200.planner.stage_planner import WorkerCaps, build_plan
    from swarm_inference_lab_b200.planner.topology import LinkProfile
    ws = [WorkerCaps("a", 1.0, 1e12), WorkerCaps("b", 1.0, 1e12), WorkerCaps("c", 1.0, 1e12)]
    links = {}
    for x in "abc":
        for y in "abc":
            if x != y:
                slow = "c" in (x, y)
                links[(x, y)] = LinkProfile(x, y, 80.0 if slow else 1.0, 5.0 if slow else 1000.0)
    plan = build_plan(8, 1e9, 1e8, 1e8, ws, links, boundary_bytes=8192, batch=1,
                      mode="speed", max_stages=2)
    assert {w for w, _, _ in plan.stages} <= {"a", "b"}


def test_engine_competition_rejects_unavailable():
    from swarm_inference_lab_b200.engines import ClusterCapabilities, EngineRegistry, RequestShape
    from swarm_inference_lab_b200.models.config import QWEN3_30B_A3B
    c = EngineRegistry().compete(QWEN3_30B_A3B, ClusterCapabilities(
        nodes={"box": {"gpus": 8, "gpu_name": "NVIDIA B200"}}), RequestShape(batch=128))
    assert c.winner is not None and c.winner.engine == "native-stage"
    assert any(name == "llama.cpp-rpc" for name, _ in c.rejected)


def test_cli_dry_run_and_inspect(tmp_path):
    from typer.testing import CliRunner
    from swarm_inference_lab_b200.cli import app
    r = CliRunner().invoke(app, ["run", "llama-3-8b-shape", "--prompt", "hi", "--dry-run", "--json",
                                 "--gpus", "8"])
    assert r.exit_code == 0, r.output
    d = json.loads(r.output.strip().splitlines()[-1])
    assert d["plan"].startswith("local:") and "terms" in d
    st = tmp_path / "st"
    r = CliRunner().invoke(app, ["cluster", "create", "lab", "--state-dir", str(st), "--json"])
    assert r.exit_code == 0, r.output
    assert json.loads(r.output)["pairing_uri"].startswith("swarm-pair://")
    r = CliRunner().invoke(app, ["cluster", "create", "lab", "--state-dir", str(st)])
    assert r.exit_code == 3


def test_cli_identity_and_service_files(tmp_path):
    """``identity create`` / ``fingerprint`` round trip (no overwrite without --force) and
    ``node install-service`` / ``uninstall-service`` (only its own unit, only with --yes)."""
    from typer.testing import CliRunner

    from swarm_inference_lab_b200.cli import app
    run = CliRunner().invoke
    idp = tmp_path / "id.json"
    r = run(app, ["identity", "create", "--name", "w7", "--out", str(idp)])
    assert r.exit_code == 0, r.output
    fp = json.loads(r.output)["fingerprint"]
    r = run(app, ["identity", "fingerprint", str(idp)])
    assert r.exit_code == 0 and r.output.strip() == fp
    assert run(app, ["identity", "create", "--out", str(idp)]).exit_code != 0
    st, unit = tmp_path / "st", tmp_path / "agent.service"
    assert run(app, ["cluster", "create", "lab", "--state-dir", str(st), "--json"]).exit_code == 0
    r = run(app, ["node", "install-service", "--state-dir", str(st), "--path", str(unit)])
    assert r.exit_code == 0 and unit.is_file()
    assert run(app, ["node", "uninstall-service", "--path", str(unit)]).exit_code != 0
    assert unit.is_file()
    other = tmp_path / "other.service"
    other.write_text("[Service]\nExecStart=/bin/true\n")
    assert run(app, ["node", "uninstall-service", "--path", str(other), "--yes"]).exit_code != 0
    assert other.is_file()
    r = run(app, ["node", "uninstall-service", "--path", str(unit), "--yes"])
    assert r.exit_code == 0 and not unit.exists()


def test_cli_topology_simulate_and_validate_run(tmp_path):
    from typer.testing import CliRunner

    from swarm_inference_lab_b200.cli import app
    run = CliRunner().invoke
    r = run(app, ["topology", "--rtt-ms", "20", "--bandwidth-mbps", "200", "--json"])
    assert r.exit_code == 0 and json.loads(r.output)["domain"] == "regional"
    r = run(app, ["topology", "--json"])
    assert json.loads(r.output)["domain"] == "unknown"
    r = run(app, ["simulate", "--requests", "8", "--json"])
    d = json.loads(r.output)
    assert r.exit_code == 0 and d["completed"] == 8 and d["tokens_per_s"] > 0
    good = {"exact_tokens": True, "messages_per_token_max": 2.0, "serial_waits_per_token_max": 2,
            "coordinator_intermediate_edges": 0, "sessions_closed_on_every_stage": True,
            "stage_errors": 0, "latency_tracks_network": True}
    ev = tmp_path / "ev.json"
    ev.write_text(json.dumps(good))
    assert run(app, ["validate-run", "stage_ring_wan", str(ev)]).exit_code == 0
    ev.write_text(json.dumps(dict(good, messages_per_token_max=3.0)))
    assert run(app, ["validate-run", "stage_ring_wan", str(ev)]).exit_code == 1


def test_cli_report_renders_evidence(tmp_path):
    from typer.testing import CliRunner

    from swarm_inference_lab_b200.cli import app
    from swarm_inference_lab_b200.testing.acceptance import check_contract, load_contract
    bench = {"metric": "m", "value": 6400.5, "unit": "tokens/s", "n_gpus": 1, "ms_per_step": 4.95,
             "ttft_ms_p50": 1190.0, "config": {"model": "llama-3-8b-shape", "parallelism": "tp1"},
             "clocks": {"sm_mhz": 1965.0}, "e2e": {"value": 6300.0}, "impl": "ours"}
    log = tmp_path / "bench.log"
    log.write_text("some text\n" + json.dumps(bench) + "\n")
    rep = check_contract(load_contract("stage_ring_wan"), {"exact_tokens": True})
    res = tmp_path / "contract.json"
    res.write_text(json.dumps(rep))
    r = CliRunner().invoke(app, ["report", str(log), str(res)])
    assert r.exit_code == 0, r.output
    assert "| ours | llama-3-8b-shape | tp1 | 1 | 6400.5 tokens/s |" in r.output
    assert "contract `stage_ring_wan`: FAIL" in r.output   # gates without evidence fail
    assert "| exact_tokens | True |" in r.output


def test_identity_trust_list_admits_and_refuses_registration(tmp_path):
    """``identity trust`` lets the coordinator admit an unpaired worker identity at
    registration; ``untrust`` removes it again; ``list-trusted`` shows the label."""
    import asyncio

    from typer.testing import CliRunner

    from swarm_inference_lab_b200.cli import app
    from swarm_inference_lab_b200.cluster.state import ClusterStateStore
    from swarm_inference_lab_b200.coordinator.service import CoordinatorCore
    from swarm_inference_lab_b200.security.identity import Identity
    run = CliRunner().invoke
    st = tmp_path / "st"
    assert run(app, ["cluster", "create", "lab", "--state-dir", str(st), "--json"]).exit_code == 0
    store = ClusterStateStore(st)
    core = CoordinatorCore(store.identity("coordinator"), cluster_store=store)
    w = Identity.generate("w9")
    idp = tmp_path / "w9.json"
    w.save(idp)
    req = {"worker_id": "w9", "fingerprint": w.fingerprint, "ring_endpoint": "127.0.0.1:1",
           "control_endpoint": "127.0.0.1:2", "capabilities": {}}

    async def register():
        try:
            await core.register(dict(req))
            return True
        except PermissionError:
            return False
        finally:
            for ag in core.agents.values():
                await ag.close()
            core.agents.clear()

    assert asyncio.run(register()) is False
    r = run(app, ["identity", "trust", str(idp), "--label", "lab box", "--state-dir", str(st)])
    assert r.exit_code == 0 and json.loads(r.output)["status"] == "trusted"
    lst = json.loads(run(app, ["identity", "list-trusted", "--state-dir", str(st)]).output)
    assert lst[w.fingerprint]["label"] == "lab box"
    assert asyncio.run(register()) is True
    r = run(app, ["identity", "untrust", w.fingerprint, "--state-dir", str(st)])
    assert r.exit_code == 0
    assert asyncio.run(register()) is False


def test_cli_node_roles(tmp_path):
    from typer.testing import CliRunner

    from swarm_inference_lab_b200.cli import app
    nodes = [{"node_id": "a", "decode_tok_s": 50.0, "memory_gb": 24, "link_ms": 1},
             {"node_id": "b", "decode_tok_s": 45.0, "memory_gb": 24, "link_ms": 1},
             {"node_id": "c", "decode_tok_s": 2.0, "memory_gb": 8, "link_ms": 80}]
    p = tmp_path / "nodes.json"
    p.write_text(json.dumps(nodes))
    r = CliRunner().invoke(app, ["experiment", "node-roles", str(p), "--model-gb", "40"])
    assert r.exit_code == 0, r.output
    roles = {x["node_id"]: x["role"] for x in json.loads(r.output)}
    assert roles["a"] == roles["b"] == "stage"       # the two fast nodes hold the model
    assert set(roles) == {"a", "b", "c"}
