"""Heterogeneous node utility, measured on one host (CPU, fp32): does a weaker node add
anything, and in which role?

    python -m swarm_inference_lab_b200.testing.heterogeneous --seconds 3 --out het.json

Three measurements, each with the planner's prediction next to what was observed:

* **Background lane.**  A primary decode lane (greedy ``generate`` of a real preset through
  the torch-rank worker backend) runs alone, then beside a background lane of integrity
  audits (the same backend recomputing claimed continuations; every fifth claim is tampered
  and must be caught).  Both are OS processes with fixed thread counts that start at the same
  instant.  Reported: primary tokens/s alone and shared, the slowdown, audited tokens/s,
  detections, and whether the lane pays (slowdown within ``max_slowdown``).
* **Node roles.**  Each node class (a thread count) measures its own decode rate alone; the
  role planner (``planner/roles.py``) assigns stage / replica / expert / idle roles from those
  rates and the nodes' memory.  The nodes given a serving role then run at once, and the
  observed aggregate divided by the planner's predicted aggregate is the capacity-normalised
  efficiency (shared cores make it < 1; the number says how far the prediction is off).
* **CPU expert host.**  A Qwen3-MoE-shaped decoder whose local expert memory holds only part
  of its experts: routing frequencies come from a calibration prompt, local and remote
  expert throughput and the link's round trip are measured (the remote is an
  ``ExpertService`` over TCP), the expert planner places every expert, and the hybrid
  placement runs on another prompt.  Reported: placements, predicted and measured time per
  forward, and the largest logit difference from all-local execution (fp32 rounding only).

Reference: si/experiments/heterogeneous_node_utility.py (Experiment 007: measured background
lane, CPU experts and role utility), si/experiments/background.py (background capacity
points), si/experiments/cpu_moe.py (hybrid CPU experts).
"""
from __future__ import annotations

import argparse
import json
import multiprocessing as mp
import time

import torch

PRESET = "tiny-llama-cpu"
PROMPT = [11, 22, 33, 44, 55, 66, 77, 88]
GEN = 8


# ---------------------------------------------------------------------------------- lanes
def _lane(role: str, threads: int, ready, go, seconds: float, q) -> None:
    """One process: ``primary`` decodes, ``audit`` checks claimed continuations.  It reports
    ready after loading and one warm-up job, and starts timing when the parent says go."""
    torch.set_num_threads(threads)
    from ..runtime.torch_rank import TorchRankBackend
    be = TorchRankBackend({"preset": PRESET, "seed": 0})
    truth = be.generate(PROMPT, GEN)["tokens"]            # also warms the process up
    ready.put(role)
    if not go.wait(timeout=300):
        return
    t0 = time.perf_counter()
    tokens = jobs = tampered = caught = 0
    while time.perf_counter() - t0 < seconds:
        if role == "primary":
            tokens += len(be.generate(PROMPT, GEN)["tokens"])
        else:
            claim = list(truth)
            if jobs % 5 == 4:
                claim[GEN // 2] = (claim[GEN // 2] + 1) % be.cfg.vocab_size
                tampered += 1
            rep = be.background("integrity_audit", {"prompt": PROMPT, "tokens": claim})
            caught += int(not rep["agreed"] and claim != truth)
            if rep["agreed"] != (claim == truth):
                raise RuntimeError("integrity audit gave the wrong verdict")
            tokens += len(claim)
        jobs += 1
    q.put({"role": role, "threads": threads, "tokens": tokens, "jobs": jobs,
           "seconds": time.perf_counter() - t0, "tampered": tampered, "caught": caught})


def _run_lanes(lanes: list[tuple[str, int]], seconds: float) -> list[dict]:
    """Run the lanes as processes that start timing together; their reports."""
    ctx = mp.get_context("spawn")
    q, ready, go = ctx.Queue(), ctx.Queue(), ctx.Event()
    procs = [ctx.Process(target=_lane, args=(role, th, ready, go, seconds, q), daemon=True)
             for role, th in lanes]
    for p in procs:
        p.start()
    out = []
    try:
        for _ in procs:
            ready.get(timeout=300)
        go.set()
        for _ in procs:
            out.append(q.get(timeout=seconds + 120))
    finally:
        go.set()
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.terminate()
                p.join(timeout=10)
    for r in out:
        r["tok_s"] = r["tokens"] / r["seconds"]
    return out


def background_lane(seconds: float = 3.0, primary_threads: int = 2, background_threads: int = 1,
                    max_slowdown: float = 0.10) -> dict:
    # alone before and after the shared run: the mean absorbs drift of the host's load
    before = _run_lanes([("primary", primary_threads)], seconds)[0]["tok_s"]
    shared = {r["role"]: r for r in _run_lanes([("primary", primary_threads),
                                                ("audit", background_threads)], seconds)}
    after = _run_lanes([("primary", primary_threads)], seconds)[0]["tok_s"]
    alone = 0.5 * (before + after)
    p, a = shared["primary"], shared["audit"]
    slowdown = 1.0 - p["tok_s"] / alone
    lost = max(alone - p["tok_s"], 0.0)
    return {"primary_alone_tok_s": alone, "primary_alone_spread": abs(before - after) / alone,
            "primary_shared_tok_s": p["tok_s"],
            "slowdown": slowdown, "audited_tok_s": a["tok_s"], "audits": a["jobs"],
            "tampered": a["tampered"], "caught": a["caught"],
            "audit_detection_complete": a["caught"] == a["tampered"],
            "audited_tokens_per_primary_token_lost": a["tok_s"] / lost if lost > 0 else None,
            "lane_pays": slowdown <= max_slowdown, "max_slowdown": max_slowdown,
            "primary_threads": primary_threads, "background_threads": background_threads}


def node_roles(thread_classes=(4, 2, 1), memory_fraction=(1.5, 1.2, 0.4),
               seconds: float = 3.0) -> dict:
    """Node i has ``thread_classes[i]`` threads and ``memory_fraction[i]`` x the model bytes."""
    from ..models.config import preset
    from ..planner.roles import NodeCaps, assign_roles
    cfg = preset(PRESET)
    model_bytes = 4.0 * _param_count(cfg)
    rates = []
    for th in thread_classes:
        rates.append(_run_lanes([("primary", th)], seconds)[0]["tok_s"])
    nodes = [NodeCaps(f"cpu{th}t-{i}", r, f * model_bytes, 0.05)
             for i, (th, r, f) in enumerate(zip(thread_classes, rates, memory_fraction))]
    roles = assign_roles(nodes, model_bytes)
    serving = [(n, r) for n, r in zip(nodes, roles) if r.role in ("stage", "replica")]
    # every serving node here holds the whole model alone, so each one is a replica
    by_id = {n.node_id: th for n, th in zip(nodes, thread_classes)}
    together = _run_lanes([("primary", by_id[r.node_id]) for _, r in serving], seconds)
    predicted = sum(r.gain_tok_s for _, r in serving)
    observed = sum(x["tok_s"] for x in together)
    return {"model_bytes": model_bytes,
            "nodes": [{"node_id": n.node_id, "threads": th, "decode_tok_s": n.decode_tok_s,
                       "memory_bytes": n.memory_bytes, "role": r.role, "gain_tok_s": r.gain_tok_s}
                      for n, th, r in zip(nodes, thread_classes, roles)],
            "predicted_aggregate_tok_s": predicted, "observed_aggregate_tok_s": observed,
            "capacity_normalised_efficiency": observed / predicted if predicted > 0 else 0.0}


def _param_count(cfg) -> int:
    H, I, V = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size
    att = H * cfg.num_heads * cfg.head_dim * 2 + H * cfg.num_kv_heads * cfg.head_dim * 2
    return cfg.num_layers * (att + 3 * H * I + 2 * H) + 2 * V * H + H


# ------------------------------------------------------------------------------ CPU experts
class _Counting:
    """Wraps a backend and counts the rows routed to every (layer, expert)."""

    def __init__(self, inner):
        self.inner, self.rows = inner, {}

    def experts(self, layer, x, ids, weights):
        for e, n in zip(*torch.unique(ids, return_counts=True)):
            self.rows[(layer, int(e))] = self.rows.get((layer, int(e)), 0) + int(n)
        return self.inner.experts(layer, x, ids, weights)


def cpu_experts(tokens: int = 16, local_fraction: float = 0.5, repeats: int = 3) -> dict:
    from ..models.reference import ReferenceDecoder, random_source
    from ..planner.expert_planner import ExpertStats, RemoteOwner, plan_experts
    from ..planner.topology import LinkProfile
    from ..runtime.expert_service import ExpertClient, ExpertStore, Microshard
    from ..runtime.moe_backends import HybridMoEBackend, LocalMoEBackend, WholeExpertRemoteBackend
    from .expert_backends import LEASE, _config, _Servers
    cfg = _config()
    get = random_source(7, std=0.1)
    I, H = cfg.moe_intermediate_size, cfg.hidden_size
    experts = [(l, e) for l in range(cfg.num_layers) for e in range(cfg.num_experts)]
    # routing frequencies come from one prompt, the placement is then run on another
    calib = torch.randint(0, cfg.vocab_size, (tokens,), generator=torch.Generator().manual_seed(5))
    ids = torch.randint(0, cfg.vocab_size, (tokens,), generator=torch.Generator().manual_seed(6))
    local, remote = ExpertStore(), ExpertStore()
    for l, e in experts:
        p = f"model.layers.{l}.mlp.experts.{e}."
        w = (get(p + "gate_proj.weight", (I, H)), get(p + "up_proj.weight", (I, H)),
             get(p + "down_proj.weight", (H, I)))
        local.add(Microshard(l, e, 0, I), *w)
        remote.add(Microshard(l, e, 0, I), *w)
    expert_bytes = 3 * I * H * 4
    srv = _Servers([remote])
    try:
        # calibration: routing frequencies per forward of the calibration prompt
        count = _Counting(LocalMoEBackend(local))
        dec = ReferenceDecoder(cfg, get)
        dec.moe_backend = count
        dec.forward(calib, dec.new_cache())
        routed = sum(count.rows.values())
        freq = dict(count.rows)
        # the all-local reference on the evaluated prompt
        dec = ReferenceDecoder(cfg, get)
        dec.moe_backend = LocalMoEBackend(local)
        ref = dec.forward(ids, dec.new_cache())
        t0 = time.perf_counter()
        for _ in range(repeats):
            dec.forward(ids, dec.new_cache())
        local_ms = (time.perf_counter() - t0) * 1e3 / repeats
        # local and remote expert throughput, and the link's round trip
        x = torch.randn(64, H, generator=torch.Generator().manual_seed(1))
        t0 = time.perf_counter()
        for _ in range(10):
            local.forward(0, 0, x)
        local_rows_per_ms = 640 / ((time.perf_counter() - t0) * 1e3)
        probe = WholeExpertRemoteBackend({(0, 0): ExpertClient("127.0.0.1", srv.ports[0])}, LEASE)
        one = torch.zeros(1, 2, dtype=torch.long)
        w1 = torch.tensor([[1.0, 0.0]])
        try:
            probe.experts(0, x[:1], one, w1)                              # connect
            t0 = time.perf_counter()
            for _ in range(20):
                probe.experts(0, x[:1], one, w1)
            rtt_ms = (time.perf_counter() - t0) * 1e3 / 20
            ids64 = torch.zeros(64, 2, dtype=torch.long)
            w64 = torch.tensor([[1.0, 0.0]]).repeat(64, 1)
            t0 = time.perf_counter()
            for _ in range(10):
                probe.experts(0, x, ids64, w64)
            batch_ms = (time.perf_counter() - t0) * 1e3 / 10
        finally:
            probe.close()
        remote_rows_per_ms = 64 * 2 / max(batch_ms - rtt_ms, 1e-3)
        link = LinkProfile("primary", "cpu-expert-host", rtt_ms=rtt_ms, bandwidth_MBps=1000.0)
        stats = [ExpertStats(l, e, freq.get((l, e), 0.0), expert_bytes) for l, e in experts]
        budget = int(local_fraction * expert_bytes * len(experts))
        decisions = plan_experts(stats, local_budget=budget, local_rows_per_ms=local_rows_per_ms,
                                 remotes=[RemoteOwner("cpu-expert-host", link, remote_rows_per_ms,
                                                      expert_bytes * len(experts))],
                                 hidden=H, act_bytes=4)
        placements = {}
        for d in decisions:
            placements[d.placement] = placements.get(d.placement, 0) + 1
        whole = WholeExpertRemoteBackend({(d.layer, d.expert): ExpertClient("127.0.0.1", srv.ports[0])
                                          for d in decisions if d.placement == "whole_remote"}, LEASE)
        try:
            hyb = HybridMoEBackend.from_decisions(decisions, local=LocalMoEBackend(local),
                                                  whole=whole, micro=None)
            dec = ReferenceDecoder(cfg, get)
            dec.moe_backend = hyb
            out = dec.forward(ids, dec.new_cache())
            t0 = time.perf_counter()
            for _ in range(repeats):
                out = dec.forward(ids, dec.new_cache())
            hybrid_ms = (time.perf_counter() - t0) * 1e3 / repeats
            remote_requests = whole.requests
        finally:
            whole.close()
    finally:
        srv.close()
    diff = (out - ref).abs().max().item()
    return {"experts": len(experts), "local_fraction": local_fraction, "routed_rows": routed,
            "placements": placements, "local_rows_per_ms": local_rows_per_ms,
            "remote_rows_per_ms": remote_rows_per_ms, "rtt_ms": rtt_ms,
            "predicted_expert_ms": sum(d.expected_ms for d in decisions),
            "all_local_ms_per_forward": local_ms, "hybrid_ms_per_forward": hybrid_ms,
            "remote_requests": remote_requests, "max_abs_logit_diff": diff, "exact": diff <= 1e-5}


def run(seconds: float = 3.0, tokens: int = 16) -> dict:
    return {"name": "heterogeneous_utility", "background_lane": background_lane(seconds),
            "node_roles": node_roles(seconds=seconds), "cpu_experts": cpu_experts(tokens)}


def markdown(rep: dict) -> str:
    b, n, c = rep["background_lane"], rep["node_roles"], rep["cpu_experts"]
    out = ["| background lane | primary alone tok/s | shared tok/s | slowdown | audited tok/s | "
           "caught / tampered | pays |", "|---|---|---|---|---|---|---|",
           f"| {b['primary_threads']} + {b['background_threads']} threads | "
           f"{b['primary_alone_tok_s']:.1f} | {b['primary_shared_tok_s']:.1f} | {b['slowdown']:.1%} | "
           f"{b['audited_tok_s']:.1f} | {b['caught']} / {b['tampered']} | {b['lane_pays']} |", "",
           "| node | threads | decode tok/s | memory / model | role | gain tok/s |",
           "|---|---|---|---|---|---|"]
    out += [f"| {x['node_id']} | {x['threads']} | {x['decode_tok_s']:.1f} | "
            f"{x['memory_bytes'] / n['model_bytes']:.1f} | {x['role']} | {x['gain_tok_s']:.1f} |"
            for x in n["nodes"]]
    out += ["", f"predicted aggregate {n['predicted_aggregate_tok_s']:.1f} tok/s, observed "
                f"{n['observed_aggregate_tok_s']:.1f} (capacity-normalised efficiency "
                f"{n['capacity_normalised_efficiency']:.2f})", "",
            "| CPU experts | placements | rtt ms | all-local ms | hybrid ms | max logit diff | exact |",
            "|---|---|---|---|---|---|---|",
            f"| {c['experts']} experts, {c['local_fraction']:.0%} local memory | "
            f"{json.dumps(c['placements'])} | {c['rtt_ms']:.2f} | {c['all_local_ms_per_forward']:.1f} | "
            f"{c['hybrid_ms_per_forward']:.1f} | {c['max_abs_logit_diff']:.1e} | {c['exact']} |"]
    return "\n".join(out)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--seconds", type=float, default=3.0)
    ap.add_argument("--tokens", type=int, default=16)
    ap.add_argument("--out", default=None)
    a = ap.parse_args(argv)
    rep = run(a.seconds, a.tokens)
    if a.out:
        with open(a.out, "w") as f:
            json.dump(rep, f, indent=1)
    print(markdown(rep))
    return 0 if rep["cpu_experts"]["exact"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
