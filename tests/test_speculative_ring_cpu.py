"""Exact speculation on the stage ring (CPU): the session controller drafts by prompt lookup,
verifies the draft in one VERIFY_CANDIDATES pass through both stages, accepts the longest
prefix equal to the greedy predictions plus one token, and rolls the stages' caches back past
rejected candidates (``truncate_to`` on the next frame).  The tokens must be exactly the
single-process greedy tokens, with fewer ring messages per token than plain decode."""
import asyncio

import torch

from swarm_inference_lab_b200.coordinator.session import Route, SessionController
from swarm_inference_lab_b200.models.config import TINY_LLAMA_CPU
from swarm_inference_lab_b200.models.reference import ReferenceDecoder, random_source
from swarm_inference_lab_b200.testing.wan_ring import _ring
from swarm_inference_lab_b200.transport.stage_ring_net import ConnectionPool

# A repeated trigram makes the first drafts come from the prompt (and be rejected, so the
# rollback path runs); later drafts come from the generated tokens.
PROMPT = [11, 12, 13, 14, 11, 12, 13, 15, 16, 11, 12]
NEW = 24


async def _decode(k: int):
    ring = await _ring(TINY_LLAMA_CPU, random_source(0))
    ctl = SessionController(Route(ring["entry"], 1, "wan-ring", "rev", ring["range0"]),
                            pool=ConnectionPool(timeout=10.0), speculate_k=k)
    toks = []
    try:
        async for ev in ctl.stream(PROMPT, NEW, f"spec{k}"):
            if ev["event"] == "token":
                toks.append(ev["token"])
        frames = sum(px.stats["request_frames"] for px in ring["proxies"])
        errors = [list(o.stats.errors) for o in ring["owners"]]
        closed = [o.stats.sessions_closed for o in ring["owners"]]
    finally:
        await ctl.pool.close()
        for o in ring["owners"]:
            await o.pool.close()
        for px in ring["proxies"]:
            await px.close()
        for s in ring["servers"]:
            await s.close()
    return toks, ctl.spec_stats, frames, errors, closed


def test_speculative_ring_decode_is_exact_and_sends_fewer_messages():
    torch.set_num_threads(2)
    expect = ReferenceDecoder(TINY_LLAMA_CPU, random_source(0)).greedy_generate(PROMPT, NEW)[0]
    plain, _, frames_plain, err0, _ = asyncio.run(_decode(0))
    spec, stats, frames_spec, err1, closed = asyncio.run(_decode(4))
    assert plain == expect
    assert spec == expect
    assert stats["verify_calls"] > 0 and stats["accepted"] > 0
    assert stats["drafted"] > stats["accepted"]        # some candidates rejected: rollback ran
    assert frames_spec < frames_plain, (frames_spec, frames_plain)
    assert err0 == [[], []] and err1 == [[], []]
    assert closed == [1, 1]


def test_speculation_through_the_coordinator_is_exact():
    """``speculate_k`` on a request submitted to the coordinator (in-process, two worker
    runtimes serving the 2-stage tiny Llama) gives the greedy tokens."""
    from swarm_inference_lab_b200.coordinator.service import CoordinatorCore, CoordinatorRpcServer
    from swarm_inference_lab_b200.runtime.worker_runtime import WorkerRuntime
    from swarm_inference_lab_b200.security.identity import Identity

    torch.set_num_threads(2)
    expect = ReferenceDecoder(TINY_LLAMA_CPU, random_source(0)).greedy_generate(PROMPT, NEW)[0]

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
            toks = [ev["token"] async for ev in core.submit_stream(
                {"model": dep["model"], "prompt_ids": PROMPT, "max_tokens": NEW, "speculate_k": 4})
                if ev["event"] == "token"]
            frames = [w.owner.stats.frames for w in ws]
            return toks, frames
        finally:
            for w in ws:
                await w.stop()
            await rpc.stop()

    toks, frames = asyncio.run(go())
    assert toks == expect
    assert frames[0] < NEW + 2  # fewer stage-0 frames than one per token (plus open / close)


def test_out_of_range_rollback_is_refused():
    """A frame whose ``truncate_to`` lies beyond the session's cache is answered with an
    ERROR frame (StageError at the controller) and leaves the session usable."""
    import pytest

    from swarm_inference_lab_b200.coordinator.session import StageError
    from swarm_inference_lab_b200.protocol import stage_ring as sr

    async def go():
        ring = await _ring(TINY_LLAMA_CPU, random_source(0))
        ctl = SessionController(Route(ring["entry"], 1, "wan-ring", "rev", ring["range0"]),
                                pool=ConnectionPool(timeout=10.0))
        try:
            await ctl._open("s1", "r1")
            tok, _ = await ctl._run_tokens("s1", "r1", PROMPT, 0, sr.Operation.PREFILL, False)
            with pytest.raises(StageError, match="truncate_to"):
                await ctl._run_tokens("s1", "r1", [tok], len(PROMPT), sr.Operation.DECODE, False,
                                      truncate_to=len(PROMPT) + 5)
            # the session still decodes from where it was
            tok2, _ = await ctl._run_tokens("s1", "r1", [tok], len(PROMPT), sr.Operation.DECODE,
                                            False)
            return tok, tok2
        finally:
            await ctl.pool.close()
            for o in ring["owners"]:
                await o.pool.close()
            for px in ring["proxies"]:
                await px.close()
            for s in ring["servers"]:
                await s.close()

    tok, tok2 = asyncio.run(go())
    expect = ReferenceDecoder(TINY_LLAMA_CPU, random_source(0)).greedy_generate(PROMPT, 2)[0]
    assert [tok, tok2] == expect


def test_speculation_turns_itself_off_when_drafts_fail(monkeypatch):
    """Drafts that are always wrong: after the warm-up verifications the controller stops
    drafting for the rest of the stream; the tokens stay exact."""
    import swarm_inference_lab_b200.coordinator.session as S

    monkeypatch.setattr(S, "prompt_lookup_draft", lambda toks, k, *a, **kw: [0] * k)
    torch.set_num_threads(2)
    expect = ReferenceDecoder(TINY_LLAMA_CPU, random_source(0)).greedy_generate(PROMPT, NEW)[0]

    async def go():
        ring = await _ring(TINY_LLAMA_CPU, random_source(0))
        ctl = SessionController(Route(ring["entry"], 1, "wan-ring", "rev", ring["range0"]),
                                pool=ConnectionPool(timeout=10.0), speculate_k=3, spec_warmup=4)
        try:
            toks = [ev["token"] async for ev in ctl.stream(PROMPT, NEW, "bad") if ev["event"] == "token"]
        finally:
            await ctl.pool.close()
            for o in ring["owners"]:
                await o.pool.close()
            for px in ring["proxies"]:
                await px.close()
            for s in ring["servers"]:
                await s.close()
        return toks, ctl.spec_stats

    toks, st = asyncio.run(go())
    assert toks == expect
    assert st["disabled"] and st["verify_calls"] == 4 and st["accepted"] == 0
