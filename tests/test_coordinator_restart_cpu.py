"""A coordinator restart (CPU, in-process): the deployed model is recorded in the durable
state; a new coordinator on the same state directory and port is told nothing, the workers
re-register through their heartbeats (their reservations for the old deployment are void),
``restore`` redeploys the model under its name with a new generation, and a request then
produces the reference tokens.  A request that was running is marked ``replay_required``;
an unloaded model is not restored."""
import asyncio

import torch

PROMPT = list(range(3, 15))


def test_restart_restores_deployed_models(tmp_path):
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
        core = CoordinatorCore(ident, state_dir=tmp_path, require_member=False,
                               heartbeat_timeout_s=30.0, heartbeat_s=0.2)
        rpc = CoordinatorRpcServer(core, host="127.0.0.1", port=0)
        port = await rpc.start()
        ws = []
        try:
            for i in range(2):
                w = WorkerRuntime(f"w{i}", Identity.generate(f"w{i}"), f"127.0.0.1:{port}",
                                  coordinator_fingerprint=ident.fingerprint, heartbeat_s=0.2,
                                  device="cpu")
                await w.start()
                ws.append(w)
            dep = await core.deploy({"model": {"preset": "tiny-llama-cpu", "seed": 0}, "stages": 2,
                                     "name": "tiny"})
            gen0 = dep["generation"]
            before = await tokens(core, "tiny")
            core.state.record_request("cut-off", PROMPT, {"max_tokens": 5})   # still running
            await rpc.stop()                                   # the coordinator goes away
            core2 = CoordinatorCore(ident, state_dir=tmp_path, require_member=False,
                                    heartbeat_timeout_s=30.0, heartbeat_s=0.2)
            rpc2 = CoordinatorRpcServer(core2, host="127.0.0.1", port=port)
            await rpc2.start()
            try:
                restored = await asyncio.wait_for(core2.restore(timeout_s=30.0, poll_s=0.1), 60)
                cut = core2.state.data["requests"]["cut-off"]["state"]
                st = core2.status()["models"]["tiny"]
                after = await tokens(core2, "tiny")
                await core2.unload({"model": "tiny"})
                core3 = CoordinatorCore(ident, state_dir=tmp_path, require_member=False)
                nothing = await core3.restore(timeout_s=1.0)
                await core3.close()
            finally:
                await rpc2.stop()
            return before, restored, st, gen0, after, nothing, cut
        finally:
            for w in ws:
                await w.stop()

    before, restored, st, gen0, after, nothing, cut = asyncio.run(go())
    assert cut == "replay_required"
    assert before == expect
    assert restored == {"tiny": "restored"}
    assert st["phase"] == "READY" and st["generation"] > gen0
    assert len(st["stages"]) == 2
    assert after == expect
    assert nothing == {}


def test_route_generations_never_repeat_across_restarts(tmp_path):
    """Generations fence stale routes: a coordinator restarted within the same second (or
    with a clock set back) continues above the last generation it handed out."""
    from swarm_inference_lab_b200.coordinator.deployment import DeploymentManager
    from swarm_inference_lab_b200.coordinator.state import DurableState, WorkerRegistry
    from swarm_inference_lab_b200.security.identity import Identity

    ident = Identity.generate("c")
    path = tmp_path / "coordinator_state.json"
    a = DeploymentManager(WorkerRegistry(), {}, ident, DurableState(path))
    seen = [a._next_generation() for _ in range(3)]
    b = DeploymentManager(WorkerRegistry(), {}, ident, DurableState(path))
    assert b._next_generation() > max(seen)
    st = DurableState(path)
    st.set_last_generation(10 ** 12)                  # as if the clock had been far ahead
    c = DeploymentManager(WorkerRegistry(), {}, ident, DurableState(path))
    assert c._next_generation() == 10 ** 12 + 1
