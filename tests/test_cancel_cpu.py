"""Cancelling a running request (CPU): an in-process coordinator and two worker runtimes
serve the 2-stage tiny Llama; after three tokens the request is cancelled through
``CoordinatorCore.cancel`` (the ``CancelRequest`` RPC of ``swarm cancel``).  The stream must
end with a ``cancelled`` event before the next token, every stage must drop the session,
and the next request on the same deployment must still produce the reference tokens."""
import asyncio

import torch

PROMPT = list(range(3, 15))


def test_cancel_stops_the_stream_and_frees_every_stage():
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
            events, rid = [], None
            async for ev in core.submit_stream({"model": dep["model"], "prompt_ids": PROMPT,
                                                "max_tokens": 32}):
                events.append(ev)
                if ev["event"] == "accepted":
                    rid = ev["request_id"]
                if ev["event"] == "token" and ev["index"] == 2:
                    assert core.cancel({"request_id": rid})["ok"]
            st = core.status()
            owners = [w.owner for w in ws]
            closed_after_cancel = [(o.stats.sessions_opened, o.stats.sessions_closed) for o in owners]
            # A second request on the same deployment runs to completion.
            toks = [ev["token"] async for ev in core.submit_stream(
                {"model": dep["model"], "prompt_ids": PROMPT, "max_tokens": 6}) if ev["event"] == "token"]
            again = core.cancel({"request_id": rid})
            return events, st, owners, toks, again, closed_after_cancel
        finally:
            for w in ws:
                await w.stop()
            await rpc.stop()

    events, st, owners, toks, again, closed_after_cancel = asyncio.run(go())
    kinds = [e["event"] for e in events]
    assert kinds[-1] == "cancelled" and "completed" not in kinds
    assert kinds.count("token") == 3 and events[-1]["tokens"] == expect[:3]
    req = next(iter(st["requests"].values()))
    assert req["state"] == "CANCELLED" and req["tokens"] == 3
    # both stages opened and dropped the cancelled session before the next request (no error)
    assert closed_after_cancel == [(1, 1), (1, 1)], closed_after_cancel
    assert all(not o.stats.errors for o in owners), [o.stats.errors for o in owners]
    assert toks == expect
    assert again["ok"] is False and again["state"] == "CANCELLED"
