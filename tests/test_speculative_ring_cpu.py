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
