"""Micro-benchmark of one expert-parallel MoE layer: fused peer-memory dispatch / combine
against the NCCL all-gather / reduce-scatter baseline.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m swarm_inference_lab_b200.parallel.ep_bench \
        [--tokens 32] [--inter 2048]

Kimi-K2 dimensions by default (hidden 7168, 384 experts, top-8 sigmoid routing with bias,
one shared expert, e4m3 128x128 weights): every rank routes its own ``--tokens`` decode
tokens; the layer runs in a CUDA graph, device-timed with events, max over ranks.  With a
small ``--inter`` the expert GEMMs shrink and the time is dominated by token movement,
which isolates the communication path.  Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=32)
    ap.add_argument("--inter", type=int, default=2048)
    ap.add_argument("--iters", type=int, default=20)
    a = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    from ..models.config import KIMI_K2
    from ..models.deepseek import MLAModel, MLAWeights
    from ..models.dense import TPInfo
    from ..ops import norm
    from ..ops.workspace import get_workspace
    from .comm import NcclComm
    from .fused_ep import FusedEPComm

    # Two layers (dense first, then one MoE layer) at K2 width; only the MoE block is timed.
    cfg = KIMI_K2.replace(num_layers=2, moe_intermediate_size=a.inter)
    w = MLAWeights.random(cfg, TPInfo(rank, world), dev, seed=1, num_layers=2)
    L = w.layers[1]
    nccl = NcclComm()
    fused = FusedEPComm(nccl, dev, max_tokens=max(a.tokens, 1), hidden=cfg.hidden_size,
                        top_k=cfg.num_experts_per_tok)
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    h0 = (torch.randn(a.tokens, cfg.hidden_size, device=dev, generator=g) * 0.5).bfloat16()
    res = {}
    for name, comm in (("nccl", nccl), ("fused", fused)):
        model = MLAModel(w, dev, comm=comm, max_positions=128)
        h = h0.clone()
        x = torch.empty_like(h)

        def body():
            h.copy_(h0)
            _, xq, xs = norm.rmsnorm_fp8(h, L.mlp_norm, cfg.rms_norm_eps, out=x)
            model.moe(L, x, xq, xs, h)
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for _ in range(3):
                body()
        torch.cuda.current_stream(dev).wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            for _ in range(a.iters):
                body()
        graph.replay()
        torch.cuda.synchronize(dev)
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        us = torch.tensor([e0.elapsed_time(e1) * 1e3 / a.iters], device=dev, dtype=torch.float64)
        dist.all_reduce(us, op=dist.ReduceOp.MAX)
        res[name] = {"us_per_layer": round(float(us.item()), 2), "out_checksum": float(h.float().sum())}
        del graph
        dist.barrier()
    get_workspace(dev).check()
    el = w.experts_local
    bytes_per_rank = el * 3 * a.inter * cfg.hidden_size + 3 * a.inter * cfg.hidden_size
    if rank == 0:
        print(json.dumps({"world": world, "tokens_per_rank": a.tokens, "inter": a.inter,
                          "experts_per_rank": el, "expert_weight_bytes_per_rank": bytes_per_rank,
                          **res}), flush=True)
    fused.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
