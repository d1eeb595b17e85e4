"""Expert execution backends compared on one MoE decoder (CPU, fp32, real SWARMEX1 TCP).

    python -m swarm_inference_lab_b200.testing.expert_backends --tokens 16 --repeats 3

A tiny Qwen3-MoE-shaped decoder runs its routed experts four ways: locally; each expert
whole on one remote expert worker; and as microshards (contiguous intermediate slices)
split over 2 and over 4 workers whose partial outputs the caller adds in shard order.  The
workers are ``ExpertService`` servers on a background event loop; the route lease is
accepted by every worker.  Per backend and timed forward of ``--tokens`` tokens:
milliseconds, expert requests and rows served remotely, and the largest logit difference from
the all-local decoder (must be fp32 rounding only).

Reference: si/experiments/experiment_009 / experiment_010 (remote whole experts,
microsharded experts with fixed-order reduction; exactness checked against local
execution) and the ``experiment microsharding`` command of si/cli.py.
"""
from __future__ import annotations

import argparse
import asyncio
import json
import threading
import time

import torch

LEASE = "expert-backends-lease"


def _config():
    from ..models.config import ModelConfig
    return ModelConfig(name="tiny-moe-cpu", family="qwen3_moe", vocab_size=512, hidden_size=64,
                       num_layers=2, num_heads=4, num_kv_heads=2, head_dim=16, intermediate_size=96,
                       qk_norm=True, num_experts=8, num_experts_per_tok=2,
                       moe_intermediate_size=48, rms_norm_eps=1e-6)


class _Servers:
    def __init__(self, stores):
        from ..runtime.expert_service import ExpertService
        self.loop = asyncio.new_event_loop()
        self.thread = threading.Thread(target=self.loop.run_forever, daemon=True)
        self.thread.start()
        self.services = [ExpertService(s) for s in stores]
        for sv in self.services:
            sv.accept_lease(LEASE)
        self.ports = [asyncio.run_coroutine_threadsafe(sv.start(), self.loop).result(10)
                      for sv in self.services]

    def close(self):
        for sv in self.services:
            asyncio.run_coroutine_threadsafe(sv.close(), self.loop).result(10)
        self.loop.call_soon_threadsafe(self.loop.stop)
        self.thread.join(5)


def run(tokens: int = 16, repeats: int = 3, seed: int = 3) -> list[dict]:
    from ..models.reference import ReferenceDecoder, random_source
    from ..runtime.expert_service import ExpertClient, ExpertStore, Microshard, split_microshards
    from ..runtime.moe_backends import (LocalMoEBackend, MicroshardRemoteBackend,
                                        WholeExpertRemoteBackend)
    cfg = _config()
    get = random_source(7, std=0.1)
    ids = torch.randint(0, cfg.vocab_size, (tokens,), generator=torch.Generator().manual_seed(seed))
    I, H = cfg.moe_intermediate_size, cfg.hidden_size
    experts = [(l, e) for l in range(cfg.num_layers) for e in range(cfg.num_experts)]

    def weights(l, e):
        p = f"model.layers.{l}.mlp.experts.{e}."
        return get(p + "gate_proj.weight", (I, H)), get(p + "up_proj.weight", (I, H)), \
            get(p + "down_proj.weight", (H, I))

    local = ExpertStore()
    whole = ExpertStore()
    micro2 = [ExpertStore() for _ in range(2)]
    micro4 = [ExpertStore() for _ in range(4)]
    for l, e in experts:
        g, u, d = weights(l, e)
        local.add(Microshard(l, e, 0, I), g, u, d)
        whole.add(Microshard(l, e, 0, I), g, u, d)
        for stores in (micro2, micro4):
            for st, sh in zip(stores, split_microshards(l, e, I, len(stores))):
                st.add(sh, g, u, d)
    srv = _Servers([whole] + micro2 + micro4)
    ports = srv.ports
    base = ReferenceDecoder(cfg, get)
    ref = base.forward(ids, base.new_cache())
    backends = {
        "local": lambda: LocalMoEBackend(local),
        "whole_remote": lambda: WholeExpertRemoteBackend(
            {k: ExpertClient("127.0.0.1", ports[0]) for k in experts}, LEASE),
        "microshard_2": lambda: MicroshardRemoteBackend(
            {k: [ExpertClient("127.0.0.1", p) for p in ports[1:3]] for k in experts}, LEASE),
        "microshard_4": lambda: MicroshardRemoteBackend(
            {k: [ExpertClient("127.0.0.1", p) for p in ports[3:7]] for k in experts}, LEASE),
    }
    rows = []
    try:
        for name, make in backends.items():
            be = make()
            try:
                dec = ReferenceDecoder(cfg, get)
                dec.moe_backend = be
                out = dec.forward(ids, dec.new_cache())     # warm-up (connections)
                rows_before = [sv.stats["rows"] for sv in srv.services]
                req_before = getattr(be, "requests", 0)
                t0 = time.perf_counter()
                for _ in range(repeats):
                    out = dec.forward(ids, dec.new_cache())
                ms = (time.perf_counter() - t0) * 1e3 / repeats
            finally:
                if hasattr(be, "close"):
                    be.close()
            served = sum(sv.stats["rows"] - r0 for sv, r0 in zip(srv.services, rows_before))
            rows.append({"backend": name, "tokens": tokens, "ms_per_forward": ms,
                         "expert_requests": (getattr(be, "requests", 0) - req_before) // repeats,
                         "remote_rows_served": served // repeats,
                         "max_abs_logit_diff": (out - ref).abs().max().item(),
                         "exact": bool((out - ref).abs().max().item() <= 1e-5)})
    finally:
        srv.close()
    return rows


def markdown(rows: list[dict]) -> str:
    out = ["| backend | ms / forward | expert requests | remote rows | max logit diff | exact |",
           "|---|---|---|---|---|---|"]
    for r in rows:
        out.append(f"| {r['backend']} | {r['ms_per_forward']:.1f} | {r['expert_requests']} | "
                   f"{r['remote_rows_served']} | {r['max_abs_logit_diff']:.2e} | {r['exact']} |")
    return "\n".join(out)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=16)
    ap.add_argument("--repeats", type=int, default=3)
    ap.add_argument("--out", default=None)
    a = ap.parse_args(argv)
    torch.set_num_threads(2)
    rows = run(a.tokens, a.repeats)
    if a.out:
        with open(a.out, "w") as f:
            json.dump(rows, f, indent=1)
    print(markdown(rows))


if __name__ == "__main__":
    main()
