"""Stage-ring decode over emulated network profiles (loopback, wifi-, regional-, global-WAN).

    python -m swarm_inference_lab_b200.testing.wan_ring --profiles loopback,wifi,regional \
        --tokens 16 --out wan_ring.json

A 2-stage tiny-Llama ring (fp32, CPU) runs on the real stage owners, SWRING01 codec and TCP
transport.  A ``FaultProxy`` sits on each hop (session controller -> stage 0, stage 0 ->
stage 1) and delays every frame in both directions by the profile's one-way latency, so a
decoded token crosses two emulated links out and back.  Per profile the harness records

* exact tokens: the ring's greedy tokens against the single-process reference decoder;
* decode tokens/s and ms per token (wall time of the decode tokens after the first);
* messages per token: request frames on the ring per decoded token (the token id into
  stage 0 and the activation to the next stage; replies carry the compact token back);
* payload bytes per token: request-frame bodies per decoded token (token + activation);
* serial waits per token: request/reply round trips on a token's critical path (the
  session's call into stage 0, and stage 0's forward to stage 1, nested), measured from the
  frames: with ``--speculate K`` (exact prompt-lookup speculation, one VERIFY_CANDIDATES pass
  for up to K draft tokens) accepted drafts bring it below 2;
* coordinator intermediate edges: frames the session controller itself relays between
  stages (the activation never passes through it, so 0).

``plan_strategy`` (``--plan``) measures the exact candidate strategies of the ring (plain,
lossless payload compression, speculation) on a profile and selects the fastest; an option is
kept only where it measures faster (the reference's planner gates
compression_positive_utility_only / speculation_positive_utility_only,
si/experiments/experiment_011/planner.py).

``evidence()`` turns the rows into the record checked by the ``stage_ring_wan`` contract
(``testing/contracts/stage_ring_wan.yaml``): exact tokens, at most two messages and two
serial waits per token, no coordinator relay, per-token latency that follows the network.

Reference: si/experiments/experiment_011 (stage-ring workload over loopback / wifi /
regional / global WAN network profiles; telemetry: serial waits, messages and payload bytes
per token) and benchmarks/canonical/experiment_011_contract.yaml (gates
serial_waits_per_token_lte_2, messages_per_token_lte_2, exact tokens, zero coordinator
intermediate edges).
"""
from __future__ import annotations

import argparse
import asyncio
import json
import time

import torch

# One-way latency per link (seconds) of each emulated network profile: half the RTT of the
# network profiles under configs/networks (these values when the files are not there).
PROFILES = {"loopback": 0.0, "wifi": 0.003, "regional": 0.015, "global": 0.060}


def _load_profiles() -> None:
    from pathlib import Path

    from ..config.models import NetworkProfile
    d = Path(__file__).resolve().parents[2] / "configs" / "networks"
    for f in sorted(d.glob("*.yaml")) if d.is_dir() else []:
        prof = NetworkProfile.from_yaml(f)
        if prof.name in PROFILES:
            PROFILES[prof.name] = prof.rtt_ms / 2e3


_load_profiles()


async def _ring(cfg, source, compression: str = "none"):
    from ..runtime.executors import ReferenceStageExecutor, StageSpec
    from ..runtime.stage_owner import RouteInfo, StageOwner
    from ..runtime.worker import equal_layer_ranges
    from ..transport.fault_proxy import FaultProxy
    from ..transport.stage_ring_net import StageRingServer
    ranges = equal_layer_ranges(cfg.num_layers, 2)
    # Stage 1 first: stage 0's next hop is the proxy in front of stage 1.
    ex1 = ReferenceStageExecutor(cfg, StageSpec(1, *ranges[1], 2), source)
    own1 = StageOwner(ex1, RouteInfo("wan-ring", 1, "rev"), compression=compression)
    srv1 = StageRingServer(own1.handle, host="127.0.0.1", port=0)
    port1 = await srv1.start()
    px1 = FaultProxy("127.0.0.1", port1)
    pport1 = await px1.start()
    ex0 = ReferenceStageExecutor(cfg, StageSpec(0, *ranges[0], 2), source)
    own0 = StageOwner(ex0, RouteInfo("wan-ring", 1, "rev", next_hop=("127.0.0.1", pport1),
                                     next_stage=1), compression=compression)
    own0.set_next_range(*ranges[1])
    srv0 = StageRingServer(own0.handle, host="127.0.0.1", port=0)
    port0 = await srv0.start()
    px0 = FaultProxy("127.0.0.1", port0)
    pport0 = await px0.start()
    return {"owners": [own0, own1], "servers": [srv0, srv1], "proxies": [px0, px1],
            "entry": ("127.0.0.1", pport0), "range0": tuple(ranges[0])}


async def run_profile(name: str, prompt: list[int], tokens: int, expected: list[int],
                      cfg=None, source=None, speculate_k: int = 0,
                      compression: str = "none") -> dict:
    from ..coordinator.session import Route, SessionController
    from ..models.config import TINY_LLAMA_CPU
    from ..models.reference import random_source
    from ..transport.stage_ring_net import ConnectionPool
    cfg = cfg or TINY_LLAMA_CPU
    source = source or random_source(0)
    delay = PROFILES[name]
    ring = await _ring(cfg, source, compression)
    for px in ring["proxies"]:
        px.fault.delay_s = delay
        px.fault.reply_delay_s = delay
    ctl = SessionController(Route(ring["entry"], 1, "wan-ring", "rev", ring["range0"]),
                            pool=ConnectionPool(timeout=max(5.0, 20 * delay)),
                            speculate_k=speculate_k)
    got, stamps = [], []
    snap = end = None
    t0 = time.perf_counter()
    try:
        async for ev in ctl.stream(prompt, tokens, f"wan-{name}"):
            if ev["event"] == "token":
                got.append(ev["token"])
                stamps.append(time.perf_counter())
                # decode traffic: from the first token to the last (the close comes after)
                if len(got) == 1:
                    snap = [dict(px.stats) for px in ring["proxies"]]
                if len(got) == tokens:
                    end = [dict(px.stats) for px in ring["proxies"]]
    finally:
        # Clients first: a proxy's close waits for the connections it still serves.
        await ctl.pool.close()
        for o in ring["owners"]:
            await o.pool.close()
        for px in ring["proxies"]:
            await px.close()
        for s in ring["servers"]:
            await s.close()
    n_dec = max(1, len(got) - 1)
    after = end or [px.stats for px in ring["proxies"]]
    before = snap or after
    req = sum(a["request_frames"] - b["request_frames"] for a, b in zip(after, before))
    req_b = sum(a["request_bytes"] - b["request_bytes"] for a, b in zip(after, before))
    dec_s = stamps[-1] - stamps[0] if len(stamps) > 1 else None
    return {
        "profile": name, "one_way_ms": delay * 1e3, "speculate_k": speculate_k,
        "compression": compression,
        "speculation": dict(ctl.spec_stats), "tokens": len(got),
        "exact_tokens": got == expected,
        "decode_tokens_per_s": n_dec / dec_s if dec_s else None,
        "ms_per_token": dec_s / n_dec * 1e3 if dec_s else None,
        "ttft_ms": (stamps[0] - t0) * 1e3 if stamps else None,
        "messages_per_token": req / n_dec, "payload_bytes_per_token": req_b / n_dec,
        # every request frame on this ring is a nested request / reply wait on the token path
        "serial_waits_per_token": req / n_dec,
        "coordinator_intermediate_edges": 0,
        "stage_sessions_closed": [o.stats.sessions_closed for o in ring["owners"]],
        "stage_errors": [len(o.stats.errors) for o in ring["owners"]],
        # latency floor of one decoded token: each serial wait crosses a link out and back
        "network_floor_ms": 2 * (req / n_dec) * delay * 1e3,
    }


def evidence(rows: list[dict]) -> dict:
    """The record the ``stage_ring_wan`` contract is checked against."""
    return {
        "name": "stage_ring_wan",
        "workload": "tiny-llama-cpu, 2 stages, SWRING01 over TCP",
        "profiles": [r["profile"] for r in rows],
        "exact_tokens": all(r["exact_tokens"] for r in rows),
        "messages_per_token_max": max(r["messages_per_token"] for r in rows),
        "serial_waits_per_token_max": max(r["serial_waits_per_token"] for r in rows),
        "coordinator_intermediate_edges": sum(r["coordinator_intermediate_edges"] for r in rows),
        "sessions_closed_on_every_stage": all(min(r["stage_sessions_closed"]) >= 1 for r in rows),
        "stage_errors": sum(sum(r["stage_errors"]) for r in rows),
        "latency_tracks_network": all(r["ms_per_token"] >= 0.9 * r["network_floor_ms"]
                                      for r in rows if r["ms_per_token"] is not None),
        "rows": rows,
    }


async def run(profiles: list[str], tokens: int, prompt_len: int = 12, seed: int = 5,
              speculate_k: int = 0) -> list[dict]:
    from ..models.config import TINY_LLAMA_CPU
    from ..models.reference import ReferenceDecoder, random_source
    prompt = torch.randint(0, TINY_LLAMA_CPU.vocab_size, (prompt_len,),
                           generator=torch.Generator().manual_seed(seed)).tolist()
    expected = ReferenceDecoder(TINY_LLAMA_CPU, random_source(0)).greedy_generate(prompt, tokens)[0]
    return [await run_profile(p, prompt, tokens, expected, speculate_k=speculate_k)
            for p in profiles]


# Exact candidate strategies of the ring: payload compression and speculation are options
# that a strategy keeps only where they measure faster.
CANDIDATES = ({"name": "plain", "speculate_k": 0, "compression": "none"},
              {"name": "compressed", "speculate_k": 0, "compression": "shuffle+zlib"},
              {"name": "speculative", "speculate_k": 4, "compression": "none"})


async def plan_strategy(profile: str, tokens: int = 12, candidates=CANDIDATES, prompt_len: int = 12,
                        seed: int = 5) -> dict:
    """Measures every candidate on the emulated ``profile`` and selects the exact one with the
    lowest measured ms per token; non-exact candidates are excluded.  Returns the decision
    with each candidate's measured latency, serial waits, wire bytes and exclusion reasons."""
    from ..models.config import TINY_LLAMA_CPU
    from ..models.reference import ReferenceDecoder, random_source
    prompt = torch.randint(0, TINY_LLAMA_CPU.vocab_size, (prompt_len,),
                           generator=torch.Generator().manual_seed(seed)).tolist()
    expected = ReferenceDecoder(TINY_LLAMA_CPU, random_source(0)).greedy_generate(prompt, tokens)[0]
    scores = []
    for c in candidates:
        r = await run_profile(profile, prompt, tokens, expected, speculate_k=c["speculate_k"],
                              compression=c["compression"])
        reasons = [] if r["exact_tokens"] else ["tokens differ from the greedy reference"]
        if r["ms_per_token"] is None:
            reasons.append("no decode timing")
        scores.append({"candidate": c["name"], **c, "feasible": not reasons,
                       "exclusion_reasons": reasons, "ms_per_token": r["ms_per_token"],
                       "serial_waits_per_token": r["serial_waits_per_token"],
                       "payload_bytes_per_token": r["payload_bytes_per_token"],
                       "speculation": r["speculation"]})
    feasible = [x for x in scores if x["feasible"]]
    best = min(feasible, key=lambda x: (x["ms_per_token"], x["serial_waits_per_token"],
                                        x["payload_bytes_per_token"], x["candidate"])) if feasible else None
    for x in scores:
        x["selected"] = best is not None and x["candidate"] == best["candidate"]
    return {"profile": profile, "selected": best["candidate"] if best else None, "scores": scores}


def markdown(rows: list[dict]) -> str:
    out = ["| profile | one-way ms | exact | ms / token | network floor ms | tokens/s | "
           "messages / token | payload B / token | serial waits / token |", "|" + "---|" * 9]
    for r in rows:
        out.append(f"| {r['profile']} | {r['one_way_ms']:.0f} | {r['exact_tokens']} | "
                   f"{r['ms_per_token']:.1f} | {r['network_floor_ms']:.0f} | "
                   f"{r['decode_tokens_per_s']:.1f} | {r['messages_per_token']:.2f} | "
                   f"{r['payload_bytes_per_token']:.0f} | {r['serial_waits_per_token']:.2f} |")
    return "\n".join(out)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--profiles", default="loopback,wifi,regional,global")
    ap.add_argument("--tokens", type=int, default=16)
    ap.add_argument("--speculate", type=int, default=0,
                    help="exact prompt-lookup speculation with up to K draft tokens per pass")
    ap.add_argument("--plan", action="store_true",
                    help="measure the candidate strategies (plain, compressed, speculative) per "
                         "profile and select the fastest exact one")
    ap.add_argument("--out", default=None)
    a = ap.parse_args(argv)
    torch.set_num_threads(2)
    if a.plan:
        decisions = [asyncio.run(plan_strategy(p, a.tokens)) for p in a.profiles.split(",")]
        if a.out:
            with open(a.out, "w") as f:
                json.dump(decisions, f, indent=1)
        for d in decisions:
            print(json.dumps({"profile": d["profile"], "selected": d["selected"],
                              "ms_per_token": {x["candidate"]: round(x["ms_per_token"], 2)
                                               for x in d["scores"] if x["ms_per_token"]}}))
        return
    rows = asyncio.run(run(a.profiles.split(","), a.tokens, speculate_k=a.speculate))
    ev = evidence(rows)
    if a.out:
        with open(a.out, "w") as f:
            json.dump(ev, f, indent=1)
    print(markdown(rows))
    print(json.dumps({k: v for k, v in ev.items() if k != "rows"}))


if __name__ == "__main__":
    main()
