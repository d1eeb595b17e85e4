"""Two-stage loopback pipeline on CPU (tiny Llama config) vs. a single process.

Gate: greedy tokens identical and per-step logits within 1e-5 of the
single-process model; restart-and-replay after injected faults yields the
same tokens with exactly one recovery.
"""
import asyncio

import pytest
import torch

from swarm_inference_lab_b200.coordinator.session import SessionController
from swarm_inference_lab_b200.models.config import TINY_LLAMA_CPU
from swarm_inference_lab_b200.models.reference import ReferenceDecoder, random_source
from swarm_inference_lab_b200.protocol import stage_ring as sr
from swarm_inference_lab_b200.testing.process_harness import LIVE, LoopbackRing
from swarm_inference_lab_b200.transport.stage_ring_net import CloseBeforeSend, ConnectionPool

PROMPT = torch.randint(0, 32000, (32,), generator=torch.Generator().manual_seed(0)).tolist()


@pytest.fixture(scope="module")
def single_process():
    torch.set_num_threads(4)
    ref = ReferenceDecoder(TINY_LLAMA_CPU, random_source(0))
    return ref.greedy_generate(PROMPT, 64)


@pytest.fixture()
def ring():
    r = LoopbackRing(stages=2, seed=0)
    r.start()
    yield r
    r.stop()
    assert not any(p.alive for p in r.procs)


def test_two_stage_matches_single_process(ring, single_process):
    toks, logits = single_process

    async def go():
        ctl = SessionController(ring.route(), return_logits=True)
        res = await ctl.generate(PROMPT, 64, request_id="exact")
        await ctl.pool.close()
        return res
    res = asyncio.run(go())
    assert res.tokens == toks
    err = max((a - b).abs().max().item() for a, b in zip(res.logits, logits))
    assert err <= 1e-5, err
    assert res.recoveries == 0


def test_socket_close_during_decode_recovers_exactly(ring, single_process):
    toks, _ = single_process
    fault = CloseBeforeSend(operation=sr.Operation.DECODE, token_position=len(PROMPT) + 1)

    async def go():
        ctl = SessionController(ring.route(), pool=ConnectionPool(fault=fault), recover=ring.recover)
        res = await ctl.generate(PROMPT, 8, request_id="drill")
        await ctl.pool.close()
        return res, ctl
    res, ctl = asyncio.run(go())
    assert fault.fired == 1
    assert res.tokens == toks[:8]
    assert res.recoveries == 1
    assert res.generations == [1, 2]
    assert any(e["event"] == "replay_complete" for e in ctl.events)


def test_worker_kill_recovers(ring, single_process):
    toks, _ = single_process

    async def go():
        ctl = SessionController(ring.route(), recover=ring.recover)
        first = await ctl.generate(PROMPT, 4, request_id="a")
        ring.procs[1].kill()  # crash the last stage between requests
        second = await ctl.generate(PROMPT, 6, request_id="b")
        await ctl.pool.close()
        return first, second
    first, second = asyncio.run(go())
    assert first.tokens == toks[:4]
    assert second.tokens == toks[:6]
    assert second.recoveries == 1


def test_stale_generation_rejected(ring):
    async def go():
        route = ring.route()
        route.generation = 0
        ctl = SessionController(route)
        try:
            await ctl.generate(PROMPT, 2, request_id="stale")
        finally:
            await ctl.pool.close()
    from swarm_inference_lab_b200.coordinator.session import StageError
    with pytest.raises(StageError, match="stale route generation"):
        asyncio.run(go())


def test_no_leaked_workers():
    assert not LIVE
