"""Stage worker process: one persistent stage owner behind a SWRING01 server.

    python -m swarm_inference_lab_b200.runtime.worker --preset tiny-llama-cpu \
        --stage 0 --stages 2 --port 0 --seed 0 [--backend reference|kernels]

Prints one JSON line ``{"ready": true, "port": P, ...}`` once listening.
The route (next hop, generation) can be (re)installed at run time with a
LOAD_STAGE control frame whose ``attributes.install_route`` carries
``{"generation": g, "next_hop": [host, port] | null, "next_layers": [a, b]}``;
older generations are rejected afterwards.

Reference: si/worker/stage_service.py:20, si/worker/process_main.py:92,
route install with lease verification si/worker/stage_runtime.py:940.
"""
from __future__ import annotations

import argparse
import asyncio
import json
import signal
import sys

import torch

from ..models.config import preset
from ..models.reference import random_source
from ..protocol import stage_ring as sr
from ..transport.stage_ring_net import StageRingServer
from .executors import KernelStageExecutor, ReferenceStageExecutor, StageSpec
from .stage_owner import RouteInfo, StageOwner


def equal_layer_ranges(num_layers: int, num_stages: int) -> list[tuple[int, int]]:
    base, rem = divmod(num_layers, num_stages)
    out, s = [], 0
    for i in range(num_stages):
        n = base + (1 if i < rem else 0)
        out.append((s, s + n))
        s += n
    return out


class Worker:
    def __init__(self, owner: StageOwner, server: StageRingServer | None = None):
        self.owner = owner
        self.server = server

    async def handle(self, msg: sr.StageMessage):
        if msg.operation == sr.Operation.LOAD_STAGE and "install_route" in msg.attributes:
            r = msg.attributes["install_route"]
            route = self.owner.route
            if int(r["generation"]) < route.generation:
                return [self.owner._reply(msg, sr.Operation.ERROR, status="ERROR",
                                          attrs={"error": "SessionError", "detail": "stale route generation"})]
            route.generation = int(r["generation"])
            route.next_hop = tuple(r["next_hop"]) if r.get("next_hop") else None
            if r.get("next_layers"):
                self.owner.set_next_range(*r["next_layers"])
                route.next_stage = self.owner.spec.stage_id + 1
            await self.owner.pool.close()
            return [self.owner._reply(msg, sr.Operation.LOAD_STAGE,
                                      attrs={"installed_generation": route.generation})]
        return await self.owner.handle(msg)


def build_owner(args) -> StageOwner:
    cfg = preset(args.preset)
    ranges = equal_layer_ranges(cfg.num_layers, args.stages)
    lo, hi = ranges[args.stage]
    spec = StageSpec(args.stage, lo, hi, args.stages)
    get = random_source(args.seed)
    if args.backend == "kernels":
        ex = KernelStageExecutor(cfg, spec, get, device="cuda")
    else:
        ex = ReferenceStageExecutor(cfg, spec, get, device="cpu", dtype=torch.float32)
    nxt = tuple(args.next.split(":")) if args.next else None
    route = RouteInfo(topology_id=args.topology, generation=args.generation,
                      model_revision=args.model_revision,
                      next_hop=(nxt[0], int(nxt[1])) if nxt else None,
                      next_stage=args.stage + 1 if args.stage + 1 < args.stages else None)
    owner = StageOwner(ex, route)
    if args.stage + 1 < args.stages:
        owner.set_next_range(*ranges[args.stage + 1])
    return owner


async def amain(args):
    owner = build_owner(args)
    w = Worker(owner)
    server = StageRingServer(w.handle, host=args.host, port=args.port)
    w.server = server
    port = await server.start()
    print(json.dumps({"ready": True, "port": port, "stage": args.stage,
                      "layers": [owner.spec.layer_start, owner.spec.layer_end]}), flush=True)
    stop = asyncio.Event()
    loop = asyncio.get_running_loop()
    for s in (signal.SIGTERM, signal.SIGINT):
        try:
            loop.add_signal_handler(s, stop.set)
        except NotImplementedError:  # pragma: no cover
            pass
    await stop.wait()
    await server.close()


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--preset", default="tiny-llama-cpu")
    ap.add_argument("--stage", type=int, required=True)
    ap.add_argument("--stages", type=int, required=True)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=0)
    ap.add_argument("--next", default="")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--generation", type=int, default=1)
    ap.add_argument("--topology", default="loopback")
    ap.add_argument("--model-revision", default="random-seed")
    ap.add_argument("--backend", choices=["reference", "kernels"], default="reference")
    args = ap.parse_args(argv)
    torch.set_num_threads(max(1, min(4, torch.get_num_threads())))
    asyncio.run(amain(args))


if __name__ == "__main__":
    sys.exit(main())
