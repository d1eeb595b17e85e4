"""Loopback replica-scaling matrix and worker fan-out timing, on the real control plane.

    python -m swarm_inference_lab_b200.testing.loopback_matrix --workers 2,4,8 \
        --concurrency 1,16,64 --stages 1 --tokens 16 --out loopback.json [--csv loopback.csv]

For every worker count N the harness starts N worker runtimes (the ``swarm node agent``
code: registration, heartbeats, gRPC worker service, SWRING01 stage server) against an
in-process coordinator, deploys the tiny fp32 Llama as N / stages replica pipelines
(cold start: stages load), then for every concurrency C submits C requests at once through
``CoordinatorCore.submit_stream`` (the replica scheduler places them) and records

* verified throughput: tokens of requests whose tokens equal the single-process greedy
  tokens of their prompt, per second of wall time (unverified tokens are not counted);
* p50 / p99 request latency and time to first token;
* per replica the number of requests it served;

and the fan-out economics of the deployment: worker registration (acquisition) time, cold
deploy time (first load of every stage), warm redeploy time (unload, then deploy the same
artifacts again), and the productive fraction of a lease of ``--lease-s`` seconds
(serving time over lease time, after the cold start).  Rows are written as JSON (and CSV),
and a markdown table is printed.

Reference: si/experiments/loopback_matrix.py:131-136 (replica scaling 2/4/8 x concurrency
1/16/64), si/experiments/worker_fanout.py (cold / warm start, acquisition, lease
economics), si/experiments/reporting.py (tables).
"""
from __future__ import annotations

import argparse
import asyncio
import csv
import json
import statistics
import time

import torch

PRESET = "tiny-llama-cpu"


async def _start_workers(n: int, target: str, coord_fp: str):
    from ..runtime.worker_runtime import WorkerRuntime
    from ..security.identity import Identity
    ws = []
    t0 = time.perf_counter()
    for i in range(n):
        w = WorkerRuntime(f"w{i:02d}", Identity.generate(f"w{i:02d}"), target,
                          coordinator_fingerprint=coord_fp, heartbeat_s=1.0, device="cpu")
        await w.start()
        ws.append(w)
    return ws, (time.perf_counter() - t0) * 1e3


def _prompts(n: int, seed: int = 0) -> list[list[int]]:
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, 32000, (8 + (i % 5),), generator=g).tolist() for i in range(n)]


async def run_cell(workers: int, concurrencies: list[int], stages: int, tokens: int,
                   lease_s: float, reference) -> list[dict]:
    from ..coordinator.service import CoordinatorCore, CoordinatorRpcServer
    from ..security.identity import Identity
    ident = Identity.generate("coordinator")
    core = CoordinatorCore(ident, require_member=False, heartbeat_timeout_s=30.0)
    rpc = CoordinatorRpcServer(core, host="127.0.0.1", port=0)
    port = await rpc.start()
    ws, acquire_ms = await _start_workers(workers, f"127.0.0.1:{port}", ident.fingerprint)
    rows = []
    try:
        replicas = max(1, workers // stages)
        model = {"preset": PRESET, "seed": 0}
        t0 = time.perf_counter()
        dep = await core.deploy({"model": model, "stages": stages, "replicas": replicas})
        cold_ms = (time.perf_counter() - t0) * 1e3
        await core.unload({"model": dep["model"]})
        t0 = time.perf_counter()
        dep = await core.deploy({"model": model, "stages": stages, "replicas": replicas,
                                 "capacity": max(concurrencies)})
        warm_ms = (time.perf_counter() - t0) * 1e3
        for conc in concurrencies:
            prompts = _prompts(conc, seed=conc)
            expect = [reference(p, tokens) for p in prompts]

            async def one(i):
                t_start = time.perf_counter()
                toks, ttft, rep = [], None, None
                async for ev in core.submit_stream({"model": dep["model"], "prompt_ids": prompts[i],
                                                    "max_tokens": tokens}):
                    if ev["event"] == "accepted":
                        rep = ev["replica"]
                    elif ev["event"] == "token":
                        if ttft is None:
                            ttft = (time.perf_counter() - t_start) * 1e3
                        toks.append(ev["token"])
                    elif ev["event"] == "failed":
                        return rep, [], None, (time.perf_counter() - t_start) * 1e3
                return rep, toks, ttft, (time.perf_counter() - t_start) * 1e3
            t0 = time.perf_counter()
            res = await asyncio.gather(*[one(i) for i in range(conc)])
            wall = time.perf_counter() - t0
            verified = sum(len(t) for (_, t, _, _), e in zip(res, expect) if t == e)
            lat = sorted(r[3] for r in res)
            ttfts = sorted(r[2] for r in res if r[2] is not None)
            per_rep: dict[str, int] = {}
            for r in res:
                per_rep[r[0]] = per_rep.get(r[0], 0) + 1
            rows.append({
                "workers": workers, "stages": stages, "replicas": replicas, "concurrency": conc,
                "tokens_per_request": tokens, "verified_requests": sum(
                    1 for (_, t, _, _), e in zip(res, expect) if t == e),
                "verified_tokens_per_s": verified / wall, "wall_s": wall,
                "latency_ms_p50": statistics.median(lat),
                "latency_ms_p99": lat[min(len(lat) - 1, int(0.99 * (len(lat) - 1) + 0.5))],
                "ttft_ms_p50": statistics.median(ttfts) if ttfts else None,
                "requests_per_replica": per_rep, "acquire_ms": acquire_ms,
                "cold_deploy_ms": cold_ms, "warm_deploy_ms": warm_ms,
                "productive_fraction": max(0.0, (lease_s - cold_ms / 1e3) / lease_s),
            })
    finally:
        for w in ws:
            await w.stop()
        await rpc.stop()
    return rows


def markdown(rows: list[dict]) -> str:
    head = ("| workers | replicas | concurrency | verified tok/s | verified req | p50 ms | p99 ms | "
            "cold deploy ms | warm deploy ms |")
    out = [head, "|" + "---|" * 9]
    for r in rows:
        out.append(f"| {r['workers']} | {r['replicas']} | {r['concurrency']} | "
                   f"{r['verified_tokens_per_s']:.1f} | {r['verified_requests']}/{r['concurrency']} | "
                   f"{r['latency_ms_p50']:.0f} | {r['latency_ms_p99']:.0f} | "
                   f"{r['cold_deploy_ms']:.0f} | {r['warm_deploy_ms']:.0f} |")
    return "\n".join(out)


def make_reference():
    from ..models.config import preset
    from ..models.reference import ReferenceDecoder, random_source
    dec = ReferenceDecoder(preset(PRESET), random_source(0))
    cache: dict = {}

    def ref(prompt, n):
        k = (tuple(prompt), n)
        if k not in cache:
            cache[k] = dec.greedy_generate(prompt, n)[0]
        return cache[k]
    return ref


async def run_matrix(workers: list[int], concurrencies: list[int], stages: int, tokens: int,
                     lease_s: float = 600.0) -> list[dict]:
    ref = make_reference()
    rows = []
    for n in workers:
        rows += await run_cell(n, concurrencies, stages, tokens, lease_s, ref)
    return rows


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--workers", default="2,4,8")
    ap.add_argument("--concurrency", default="1,16,64")
    ap.add_argument("--stages", type=int, default=1)
    ap.add_argument("--tokens", type=int, default=16)
    ap.add_argument("--lease-s", type=float, default=600.0)
    ap.add_argument("--out", default="loopback_matrix.json")
    ap.add_argument("--csv", default=None)
    a = ap.parse_args(argv)
    torch.set_num_threads(2)
    rows = asyncio.run(run_matrix([int(x) for x in a.workers.split(",")],
                                  [int(x) for x in a.concurrency.split(",")], a.stages, a.tokens,
                                  a.lease_s))
    with open(a.out, "w") as f:
        json.dump(rows, f, indent=1)
    if a.csv:
        keys = [k for k in rows[0] if k != "requests_per_replica"]
        with open(a.csv, "w", newline="") as f:
            w = csv.DictWriter(f, fieldnames=keys, extrasaction="ignore")
            w.writeheader()
            w.writerows(rows)
    print(markdown(rows))


if __name__ == "__main__":
    main()
