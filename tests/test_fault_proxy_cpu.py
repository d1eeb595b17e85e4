"""Host-side fault injection on the stage ring: a TCP ``FaultProxy`` between the
coordinator and stage 0 of an in-process 2-stage tiny-Llama ring (fp32 CPU).

Each fault (WAN delay, corrupted reply frame, swallowed frame, disconnect) is recorded in
the proxy's events; the session controller turns the three failures into one
restart-and-replay under the next route generation and still produces the single-process
greedy tokens."""
import asyncio

import pytest
import torch

from swarm_inference_lab_b200.coordinator.session import Route, SessionController
from swarm_inference_lab_b200.models.config import TINY_LLAMA_CPU
from swarm_inference_lab_b200.models.reference import ReferenceDecoder, random_source
from swarm_inference_lab_b200.runtime.executors import ReferenceStageExecutor, StageSpec
from swarm_inference_lab_b200.runtime.stage_owner import RouteInfo, StageOwner
from swarm_inference_lab_b200.runtime.worker import equal_layer_ranges
from swarm_inference_lab_b200.transport.fault_proxy import FaultProxy
from swarm_inference_lab_b200.transport.stage_ring_net import ConnectionPool, StageRingServer

PROMPT = torch.randint(0, 32000, (12,), generator=torch.Generator().manual_seed(5)).tolist()
NEW = 8


@pytest.fixture(scope="module")
def expected():
    torch.set_num_threads(2)
    return ReferenceDecoder(TINY_LLAMA_CPU, random_source(0)).greedy_generate(PROMPT, NEW)[0]


async def _ring():
    ranges = equal_layer_ranges(TINY_LLAMA_CPU.num_layers, 2)
    owners, servers, ports = [], [], []
    for i in (1, 0):  # last stage first: stage 0 needs its next hop's port
        spec = StageSpec(i, *ranges[i], 2)
        ex = ReferenceStageExecutor(TINY_LLAMA_CPU, spec, random_source(0))
        nxt = ("127.0.0.1", ports[0]) if i == 0 else None
        own = StageOwner(ex, RouteInfo("proxy-ring", 1, "rev", next_hop=nxt,
                                       next_stage=1 if i == 0 else None))
        if i == 0:
            own.set_next_range(*ranges[1])
        srv = StageRingServer(own.handle, host="127.0.0.1", port=0)
        ports.insert(0, await srv.start())
        owners.insert(0, own)
        servers.insert(0, srv)
    return owners, servers, ports, ranges


async def _run(fault: str, expected):
    owners, servers, ports, ranges = await _ring()
    proxy = FaultProxy("127.0.0.1", ports[0])
    pport = await proxy.start()
    gen = [1]

    async def recover(route, exc):
        proxy.reconnect()
        gen[0] += 1
        for o in owners:
            o.route.generation = gen[0]
        return Route(("127.0.0.1", pport), gen[0], "proxy-ring", "rev", tuple(ranges[0]))

    ctl = SessionController(Route(("127.0.0.1", pport), 1, "proxy-ring", "rev", tuple(ranges[0])),
                            pool=ConnectionPool(timeout=1.0), recover=recover)
    tokens = []
    try:
        async for ev in ctl.stream(PROMPT, NEW, "r"):
            if ev["event"] == "token":
                tokens.append(ev["token"])
                if len(tokens) == 3:
                    if fault == "delay":
                        proxy.fault.delay_s = 0.02
                    elif fault == "corrupt":
                        proxy.fault.corrupt_next = True
                    elif fault == "timeout":
                        proxy.fault.timeout_next = True
                    elif fault == "disconnect":
                        proxy.disconnect()
    finally:
        await ctl.pool.close()
        await proxy.close()
        for s in servers:
            await s.close()
        for o in owners:
            await o.pool.close()
    return tokens, proxy.events, gen[0]


@pytest.mark.parametrize("fault,kind,recoveries", [
    ("delay", "emulated_wan_delay", 0),
    ("corrupt", "emulated_corrupt_frame", 1),
    ("timeout", "emulated_timeout", 1),
    ("disconnect", "emulated_disconnection", 1),
])
def test_fault_proxy(fault, kind, recoveries, expected):
    tokens, events, gen = asyncio.run(_run(fault, expected))
    assert tokens == expected
    assert any(e["type"] == kind for e in events), events
    assert gen == 1 + recoveries
