"""Generation stops after an EOS / stop token (CPU): the checkpoint's ``eos_token_id`` comes
from ``generation_config.json`` over ``config.json``; a request through the coordinator ends
with the stop token as its last token (``stop_reason: stop_token``), every stage closes the
session, and ``ignore_eos`` runs to ``max_tokens``."""
import asyncio
import json

import torch

PROMPT = list(range(3, 15))


def test_eos_ids_from_config_and_generation_config(tmp_path):
    from swarm_inference_lab_b200.model_io.loader import checkpoint_config
    from swarm_inference_lab_b200.models.config import eos_ids
    assert eos_ids(None) == () and eos_ids(7) == (7,) and eos_ids([9, 2, 9]) == (2, 9)
    cfg = {"model_type": "llama", "hidden_size": 64, "num_attention_heads": 4, "vocab_size": 100,
           "num_hidden_layers": 2, "intermediate_size": 96, "eos_token_id": 2}
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    assert checkpoint_config(tmp_path).eos_token_ids == (2,)
    (tmp_path / "generation_config.json").write_text(json.dumps({"eos_token_id": [5, 3]}))
    assert checkpoint_config(tmp_path).eos_token_ids == (3, 5)


def test_coordinator_stream_ends_at_a_stop_token():
    from swarm_inference_lab_b200.coordinator.service import CoordinatorCore, CoordinatorRpcServer
    from swarm_inference_lab_b200.models.config import preset
    from swarm_inference_lab_b200.models.reference import ReferenceDecoder, random_source
    from swarm_inference_lab_b200.runtime.worker_runtime import WorkerRuntime
    from swarm_inference_lab_b200.security.identity import Identity

    torch.set_num_threads(2)
    expect = ReferenceDecoder(preset("tiny-llama-cpu"), random_source(0)).greedy_generate(PROMPT, 8)[0]
    stop = expect[3]
    cut = expect.index(stop) + 1

    async def run(core, name, **kw):
        evs = [ev async for ev in core.submit_stream(
            {"model": name, "prompt_ids": PROMPT, "max_tokens": 8, **kw})]
        return [e["token"] for e in evs if e["event"] == "token"], evs[-1]

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
            name = dep["model"]
            stopped = await run(core, name, stop_token_ids=[stop])
            stats = [(w.owner.stats.sessions_opened, w.owner.stats.sessions_closed) for w in ws]
            # the deployment's own EOS list, and ignore_eos
            core.models[name].eos_token_ids = (stop,)
            eos = await run(core, name)
            full = await run(core, name, ignore_eos=True)
            reasons = sorted(r["stop_reason"] for r in core.status()["requests"].values())
            return stopped, stats, eos, full, [w.owner.stats.errors for w in ws], reasons
        finally:
            for w in ws:
                await w.stop()
            await rpc.stop()

    stopped, stats, eos, full, errors, reasons = asyncio.run(go())
    assert reasons == ["length", "stop_token", "stop_token"]
    assert stopped[0] == expect[:cut] and stopped[1]["stop_reason"] == "stop_token"
    assert stopped[1]["event"] == "completed"
    assert stats == [(1, 1), (1, 1)]
    assert eos[0] == expect[:cut] and eos[1]["stop_reason"] == "stop_token"
    assert full[0] == expect and full[1]["stop_reason"] == "length"
    assert all(not e for e in errors), errors
