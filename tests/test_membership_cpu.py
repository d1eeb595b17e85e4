"""Membership changes on a running deployment (CPU): an in-process coordinator and three
worker runtimes serve the 2-stage tiny Llama with two spares.  A stage worker that leaves
gracefully (``NodeLeave``) is refused while its replica has a running request, then leaves:
its stage moves to a spare under a new generation and the next request still produces the
reference tokens.  ``RemoveWorker`` (``cluster revoke``) moves the other stage to the last
spare; with no spare left it is refused and nothing changes.  The topology view reports
coverage before and after."""
import asyncio

import torch

PROMPT = list(range(3, 15))


def test_leave_remove_and_topology():
    from swarm_inference_lab_b200.coordinator.service import CoordinatorCore, CoordinatorRpcServer
    from swarm_inference_lab_b200.models.config import preset
    from swarm_inference_lab_b200.models.reference import ReferenceDecoder, random_source
    from swarm_inference_lab_b200.runtime.worker_runtime import WorkerRuntime
    from swarm_inference_lab_b200.security.identity import Identity

    torch.set_num_threads(2)
    expect = ReferenceDecoder(preset("tiny-llama-cpu"), random_source(0)).greedy_generate(PROMPT, 5)[0]

    async def tokens(core, name):
        return [ev["token"] async for ev in core.submit_stream(
            {"model": name, "prompt_ids": PROMPT, "max_tokens": 5}) if ev["event"] == "token"]

    async def go():
        ident = Identity.generate("coordinator")
        core = CoordinatorCore(ident, require_member=False, heartbeat_timeout_s=30.0)
        rpc = CoordinatorRpcServer(core, host="127.0.0.1", port=0)
        port = await rpc.start()
        ws = {}
        out = {}
        try:
            for i in range(4):
                w = WorkerRuntime(f"w{i}", Identity.generate(f"w{i}"), f"127.0.0.1:{port}",
                                  coordinator_fingerprint=ident.fingerprint, heartbeat_s=0.2,
                                  device="cpu")
                await w.start()
                ws[f"w{i}"] = w
            dep = await core.deploy({"model": {"preset": "tiny-llama-cpu", "seed": 0}, "stages": 2})
            name = dep["model"]
            stage_workers = [s["worker_id"] for s in dep["stages"]]
            spares = [w for w in ws if w not in stage_workers]
            out["topo0"] = core.topology()
            leaver = stage_workers[1]
            # a running request on the replica blocks a graceful leave
            agen = core.submit_stream({"model": name, "prompt_ids": PROMPT, "max_tokens": 5})
            first = [await agen.__anext__(), await agen.__anext__()]      # accepted, token 0
            out["refused"] = await ws[leaver].leave()
            out["rest"] = first + [ev async for ev in agen]
            gen0 = core.models[name].deployment.generation
            out["left"] = await ws[leaver].leave()
            out["gen_after_leave"] = core.models[name].deployment.generation > gen0
            out["stages_after_leave"] = [sp.worker_id for sp in core.models[name].deployment.stages]
            out["spares"], out["leaver"] = spares, leaver
            out["tokens_after_leave"] = await tokens(core, name)
            await asyncio.sleep(0.6)                                     # heartbeats stop
            out["hb_stopped"] = not ws[leaver].registered and leaver not in core.registry.workers
            out["topo1"] = core.topology()
            # removal moves stage 0 to the last spare; the request after it is still exact
            out["removed"] = await core.remove_worker({"worker_id": stage_workers[0]})
            out["tokens_after_remove"] = await tokens(core, name)
            out["stages_after_remove"] = [sp.worker_id for sp in core.models[name].deployment.stages]
            # no spare left: removing a stage worker is refused and nothing changes
            before = [sp.worker_id for sp in core.models[name].deployment.stages]
            out["remove_refused"] = await core.remove_worker({"worker_id": before[0]})
            out["unchanged"] = before == [sp.worker_id for sp in core.models[name].deployment.stages]
            out["unknown"] = await core.remove_worker({"worker_id": "nobody"})
            return out
        finally:
            for w in ws.values():
                await w.stop()
            await rpc.stop()

    out = asyncio.run(go())
    t0 = out["topo0"]
    m0 = next(iter(t0["models"].values()))
    assert m0["complete"] and m0["layers"] == 4
    assert [s["layers"] for s in next(iter(m0["replicas"].values()))["stages"]] == [[0, 2], [2, 4]]
    assert out["refused"]["ok"] is False and "running requests" in out["refused"]["reason"]
    kinds = [e["event"] for e in out["rest"]]
    assert kinds[-1] == "completed" and [e["token"] for e in out["rest"] if e["event"] == "token"] == expect
    assert out["left"]["ok"] and out["gen_after_leave"]
    taken = out["stages_after_leave"][1]
    assert taken in out["spares"] and out["tokens_after_leave"] == expect
    assert out["left"]["moved"][0]["stages"][1] == [1, taken]
    assert out["hb_stopped"]
    m1 = next(iter(out["topo1"]["models"].values()))
    assert m1["complete"] and out["topo1"]["departed"] == [out["leaver"]]
    assert len(out["topo1"]["workers"]) == 3
    last = next(w for w in out["spares"] if w != taken)
    assert out["removed"]["ok"] and out["stages_after_remove"] == [last, taken]
    assert out["tokens_after_remove"] == expect
    assert out["remove_refused"]["ok"] is False and "no spare" in out["remove_refused"]["reason"]
    assert out["unchanged"]
    assert out["unknown"]["ok"] is False


def test_scale_replicas_up_and_down():
    """``ScaleModel``: 1 -> 2 replicas on free workers (concurrent requests then use both,
    tokens exact), 2 -> 3 refused for lack of workers with nothing changed, 2 -> 1 unloads an
    idle replica."""
    from swarm_inference_lab_b200.coordinator.service import CoordinatorCore, CoordinatorRpcServer
    from swarm_inference_lab_b200.models.config import preset
    from swarm_inference_lab_b200.models.reference import ReferenceDecoder, random_source
    from swarm_inference_lab_b200.runtime.worker_runtime import WorkerRuntime
    from swarm_inference_lab_b200.security.identity import Identity

    torch.set_num_threads(2)
    expect = ReferenceDecoder(preset("tiny-llama-cpu"), random_source(0)).greedy_generate(PROMPT, 5)[0]

    async def one(core, name):
        rep, toks = None, []
        async for ev in core.submit_stream({"model": name, "prompt_ids": PROMPT, "max_tokens": 5}):
            if ev["event"] == "accepted":
                rep = ev["replica"]
            elif ev["event"] == "token":
                toks.append(ev["token"])
        return rep, toks

    async def go():
        ident = Identity.generate("coordinator")
        core = CoordinatorCore(ident, require_member=False, heartbeat_timeout_s=30.0)
        rpc = CoordinatorRpcServer(core, host="127.0.0.1", port=0)
        port = await rpc.start()
        ws, out = [], {}
        try:
            for i in range(4):
                w = WorkerRuntime(f"w{i}", Identity.generate(f"w{i}"), f"127.0.0.1:{port}",
                                  coordinator_fingerprint=ident.fingerprint, heartbeat_s=1.0,
                                  device="cpu")
                await w.start()
                ws.append(w)
            dep = await core.deploy({"model": {"preset": "tiny-llama-cpu", "seed": 0}, "stages": 2,
                                     "capacity": 1})
            name = dep["model"]
            out["up"] = await core.scale({"model": name, "replicas": 2})
            out["both"] = await asyncio.gather(one(core, name), one(core, name))
            out["too_many"] = await core.scale({"model": name, "replicas": 3})
            out["after_refusal"] = len(core.models[name].replicas)
            out["down"] = await core.scale({"model": name, "replicas": 1})
            out["left"] = sorted(core.models[name].replicas)
            out["single"] = await one(core, name)
            out["topo"] = core.topology()
            return out
        finally:
            for w in ws:
                await w.stop()
            await rpc.stop()

    out = asyncio.run(go())
    assert out["up"] == {"ok": True, "replicas": 2, "added": ["replica1"]}
    (ra, ta), (rb, tb) = out["both"]
    assert {ra, rb} == {"replica0", "replica1"} and ta == tb == expect
    assert out["too_many"]["ok"] is False and out["after_refusal"] == 2
    assert out["down"]["ok"] and out["down"]["replicas"] == 1 and len(out["left"]) == 1
    assert out["single"][1] == expect
    m = next(iter(out["topo"]["models"].values()))
    assert m["complete"] and list(m["replicas"]) == out["left"]


def test_unreachable_worker_gets_no_stage():
    """A worker whose advertised control endpoint does not answer the coordinator registers,
    is reported unreachable, gets no stage in a plan and is never a spare; a reachable
    worker's round trip is recorded."""
    from swarm_inference_lab_b200.coordinator.service import CoordinatorCore, CoordinatorRpcServer
    from swarm_inference_lab_b200.runtime.worker_runtime import WorkerRuntime
    from swarm_inference_lab_b200.security.identity import Identity

    async def go():
        ident = Identity.generate("coordinator")
        core = CoordinatorCore(ident, require_member=False, heartbeat_timeout_s=30.0)
        rpc = CoordinatorRpcServer(core, host="127.0.0.1", port=0)
        port = await rpc.start()
        ws = []
        try:
            for i in range(2):
                w = WorkerRuntime(f"w{i}", Identity.generate(f"w{i}"), f"127.0.0.1:{port}",
                                  coordinator_fingerprint=ident.fingerprint, heartbeat_s=1.0,
                                  device="cpu")
                await w.start()
                ws.append(w)
            ghost = Identity.generate("ghost")
            rep = await core.register({"worker_id": "ghost", "fingerprint": ghost.fingerprint,
                                       "ring_endpoint": "127.0.0.1:9", "control_endpoint": "127.0.0.1:9",
                                       "capabilities": {}})
            plan = core.plan({"preset": "tiny-llama-cpu", "seed": 0}, 2)
            topo = core.topology()
            hb = await core.heartbeat({"worker_id": "ghost", "fingerprint": ghost.fingerprint})
            listed = {w["worker_id"]: w for w in core.workers()}
            assert listed["ghost"]["reachable"] is False and listed["w1"]["rtt_ms"] > 0
            return rep, plan, topo, hb, core.deployer.excluded
        finally:
            for w in ws:
                await w.stop()
            await rpc.stop()

    rep, plan, topo, hb, excluded = asyncio.run(go())
    assert rep["accepted"] and rep["reachable"] is False
    assert {p["worker_id"] for p in plan} == {"w0", "w1"}
    by = {w["worker_id"]: w for w in topo["workers"]}
    assert by["ghost"]["reachable"] is False and by["w0"]["reachable"] is True
    assert by["w0"]["link"] is not None and by["w0"]["link"]["rtt_ms"] > 0
    assert hb["ok"] and "ghost" in excluded


def test_cluster_topology_wait_polls_until_coverage(monkeypatch):
    """``cluster topology --wait`` polls the coordinator until every deployed model (and the
    named one) is covered; without coverage in time it exits 1."""
    import json

    from typer.testing import CliRunner

    import swarm_inference_lab_b200.cli as cli

    class Fake:
        def __init__(self, complete_after):
            self.calls, self.after = 0, complete_after

        async def topology(self):
            self.calls += 1
            ok = self.calls > self.after
            return {"workers": [], "departed": [], "draining": [],
                    "models": {"m": {"layers": 4, "replicas": {}, "complete": ok}} if ok or self.calls > 1 else {}}

    def with_fake(fake):
        def run(state, fn):
            import asyncio
            return asyncio.run(fn(fake))
        return run

    fake = Fake(complete_after=3)
    monkeypatch.setattr(cli, "_with_coordinator", with_fake(fake))
    r = CliRunner().invoke(cli.app, ["cluster", "topology", "--wait", "10", "--model", "m"])
    assert r.exit_code == 0, r.output
    assert fake.calls == 4 and json.loads(r.output)["models"]["m"]["complete"]
    slow = Fake(complete_after=10 ** 6)
    monkeypatch.setattr(cli, "_with_coordinator", with_fake(slow))
    r = CliRunner().invoke(cli.app, ["cluster", "topology", "--wait", "0.6", "--model", "m"])
    assert r.exit_code == 1 and slow.calls >= 2


def test_worker_metrics_through_the_coordinator():
    """``Metrics`` with ``workers``: every worker's stage view (layers, frames, tokens) and
    metrics snapshot, gathered by the coordinator after a request."""
    from swarm_inference_lab_b200.coordinator.service import (CoordinatorClient, CoordinatorCore,
                                                              CoordinatorRpcServer)
    from swarm_inference_lab_b200.runtime.worker_runtime import WorkerRuntime
    from swarm_inference_lab_b200.security.identity import Identity

    async def go():
        ident = Identity.generate("coordinator")
        core = CoordinatorCore(ident, require_member=False, heartbeat_timeout_s=30.0)
        rpc = CoordinatorRpcServer(core, host="127.0.0.1", port=0)
        port = await rpc.start()
        ws = []
        try:
            for i in range(2):
                w = WorkerRuntime(f"w{i}", Identity.generate(f"w{i}"), f"127.0.0.1:{port}",
                                  coordinator_fingerprint=ident.fingerprint, heartbeat_s=1.0,
                                  device="cpu")
                await w.start()
                ws.append(w)
            dep = await core.deploy({"model": {"preset": "tiny-llama-cpu", "seed": 0}, "stages": 2})
            _ = [ev async for ev in core.submit_stream(
                {"model": dep["model"], "prompt_ids": PROMPT, "max_tokens": 3})]
            cli = CoordinatorClient(f"127.0.0.1:{port}")
            try:
                rep = await cli.metrics(workers=True)
                plain = await cli.metrics()
            finally:
                await cli.close()
            return rep, plain
        finally:
            for w in ws:
                await w.stop()
            await rpc.stop()

    rep, plain = asyncio.run(go())
    assert "workers" not in plain and "coordinator_tokens" in str(plain["snapshot"])
    ws = rep["workers"]
    assert set(ws) == {"w0", "w1"}
    layers = sorted(tuple(w["stage"]["layers"]) for w in ws.values())
    assert layers == [(0, 2), (2, 4)]
    assert all(w["stage"]["frames"] > 0 for w in ws.values())
    assert all(isinstance(w["metrics"], dict) for w in ws.values())


def test_drain_lets_running_requests_finish():
    """``drain`` (the coordinator's shutdown): a request already streaming runs to completion,
    a new one is refused, and drain returns once nothing runs."""
    from swarm_inference_lab_b200.coordinator.service import CoordinatorCore, CoordinatorRpcServer
    from swarm_inference_lab_b200.models.config import preset
    from swarm_inference_lab_b200.models.reference import ReferenceDecoder, random_source
    from swarm_inference_lab_b200.runtime.worker_runtime import WorkerRuntime
    from swarm_inference_lab_b200.security.identity import Identity

    torch.set_num_threads(2)
    expect = ReferenceDecoder(preset("tiny-llama-cpu"), random_source(0)).greedy_generate(PROMPT, 6)[0]

    async def go():
        ident = Identity.generate("coordinator")
        core = CoordinatorCore(ident, require_member=False, heartbeat_timeout_s=30.0)
        rpc = CoordinatorRpcServer(core, host="127.0.0.1", port=0)
        port = await rpc.start()
        ws = []
        try:
            for i in range(2):
                w = WorkerRuntime(f"w{i}", Identity.generate(f"w{i}"), f"127.0.0.1:{port}",
                                  coordinator_fingerprint=ident.fingerprint, heartbeat_s=1.0,
                                  device="cpu")
                await w.start()
                ws.append(w)
            dep = await core.deploy({"model": {"preset": "tiny-llama-cpu", "seed": 0}, "stages": 2})
            agen = core.submit_stream({"model": dep["model"], "prompt_ids": PROMPT, "max_tokens": 6})
            first = [await agen.__anext__(), await agen.__anext__()]        # accepted, token 0
            drain = asyncio.get_running_loop().create_task(core.drain(30.0))
            await asyncio.sleep(0.05)
            refused = [ev async for ev in core.submit_stream(
                {"model": dep["model"], "prompt_ids": PROMPT, "max_tokens": 2})]
            rest = [ev async for ev in agen]
            left = await drain
            return first + rest, refused, left
        finally:
            for w in ws:
                await w.stop()
            await rpc.stop()

    evs, refused, left = asyncio.run(go())
    assert evs[-1]["event"] == "completed"
    assert [e["token"] for e in evs if e["event"] == "token"] == expect
    assert refused[-1]["event"] == "failed" and "shutting down" in refused[-1]["error"]
    assert left == 0


def test_cli_scale_and_metrics_commands(monkeypatch):
    """``model scale`` exits 1 when the coordinator cannot make the change; ``metrics
    --prometheus`` prints the text exposition and ``--workers`` asks for the worker views."""
    import json

    from typer.testing import CliRunner

    import swarm_inference_lab_b200.cli as cli

    calls = []

    class Fake:
        async def scale(self, name, replicas):
            calls.append(("scale", name, replicas))
            return {"ok": replicas <= 2, "replicas": min(replicas, 2)}

        async def metrics(self, *, workers=False):
            calls.append(("metrics", workers))
            rep = {"snapshot": {"coordinator_tokens": 5}, "prometheus": "coordinator_tokens 5\n"}
            if workers:
                rep["workers"] = {"w0": {"stage": {"frames": 3}, "metrics": {}}}
            return rep

    def run_with(state, fn):
        import asyncio
        return asyncio.run(fn(Fake()))

    monkeypatch.setattr(cli, "_with_coordinator", run_with)
    invoke = CliRunner().invoke
    assert invoke(cli.app, ["model", "scale", "m", "--replicas", "2"]).exit_code == 0
    assert invoke(cli.app, ["model", "scale", "m", "--replicas", "5"]).exit_code == 1
    r = invoke(cli.app, ["metrics", "--prometheus"])
    assert r.exit_code == 0 and r.output.startswith("coordinator_tokens 5")
    r = invoke(cli.app, ["metrics", "--workers"])
    assert json.loads(r.output)["workers"]["w0"]["stage"]["frames"] == 3
    assert calls == [("scale", "m", 2), ("scale", "m", 5), ("metrics", False), ("metrics", True)]
