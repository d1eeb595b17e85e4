"""Multi-GPU expert-parallel self-test of the MLA (DeepSeek-V3 / Kimi-K2) model.

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m swarm_inference_lab_b200.parallel.ep_selftest

Every rank serves its own sequences (data-parallel attention).  Each rank runs
them with the full model on its own GPU (EP=1), then with the experts sharded
over all ranks (EP=world) through the NCCL path (all-gather, local experts,
reduce-scatter) and through the fused peer-memory path (decode steps: e4m3
dispatch, combine fused into the down projection).  Logits must agree.
Rank 0 prints one JSON line.  The process group has a short timeout.
"""
from __future__ import annotations

import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    from ..engine.kv_cache import PagedKVCache
    from ..models.config import preset
    from ..models.deepseek import MLAModel, MLAWeights
    from ..models.dense import ForwardBatch, TPInfo
    from ..ops.workspace import get_workspace
    from .comm import LocalComm, NcclComm
    from .fused_ep import FusedEPComm

    cfg = preset(os.environ.get("SIL_SELFTEST_MODEL", "tiny-mla-gpu"))
    if cfg.num_experts % world:
        cfg = cfg.replace(num_experts=world * max(1, cfg.num_experts // world))
    B, P = 2, 90
    nccl = NcclComm()
    g = torch.Generator().manual_seed(100 + rank)   # each rank its own sequences
    ids = torch.randint(0, cfg.vocab_size, (B, P), generator=g)

    def run(ep, comm, forced=None):
        w = MLAWeights.random(cfg, ep, dev, seed=11)
        model = MLAModel(w, dev, comm=comm, max_positions=1024)
        pages = (P + 8 + 63) // 64
        kv = PagedKVCache(model.num_layers, 1, B * pages, dev, latent_dim=model.latent_dim)
        bt = torch.arange(B * pages, dtype=torch.int32, device=dev).view(B, pages)
        flat = ids.reshape(-1).to(dev)
        pos = torch.arange(P, dtype=torch.int32, device=dev).repeat(B)
        slots = (bt[:, :1] * 64).repeat(1, P).reshape(-1) + pos
        fb = ForwardBatch(ids=flat, positions=pos, slots=slots.int(),
                          seq_lens=torch.full((B,), P, dtype=torch.int32, device=dev),
                          block_table=bt, last_idx=torch.arange(B, device=dev) * P + P - 1,
                          is_decode=False,
                          cu_q=torch.arange(0, B * P + 1, P, dtype=torch.int32, device=dev),
                          max_q_len=P)
        logits = [model.logits(model.forward_hidden(fb, kv), fb)]
        toks = [model.greedy(logits[0])]
        tok = forced[0] if forced else toks[0]
        for s in range(3):
            p = P + s
            fbd = ForwardBatch(ids=tok, positions=torch.full((B,), p, dtype=torch.int32, device=dev),
                               slots=(bt[:, 0] * 64 + p).int(),
                               seq_lens=torch.full((B,), p + 1, dtype=torch.int32, device=dev),
                               block_table=bt, last_idx=torch.arange(B, device=dev), is_decode=True,
                               decode_splits=2)
            lg = model.logits(model.forward_hidden(fbd, kv), fbd)
            logits.append(lg)
            toks.append(model.greedy(lg))
            tok = forced[s + 1] if forced else toks[-1]
        torch.cuda.synchronize()
        return logits, toks

    def rel_rows(a, b):
        return ((a - b).norm(dim=1) / (a.norm(dim=1) + 1e-6))

    # Teacher-forced: every run consumes the EP=1 run's tokens, so a near-tie flip in one
    # greedy choice cannot make later steps incomparable.
    full, full_toks = run(TPInfo(), LocalComm())
    fused = FusedEPComm(nccl, dev, max_tokens=64, hidden=cfg.hidden_size,
                        top_k=cfg.num_experts_per_tok)
    res = {}
    for name, comm in (("nccl", nccl), ("fused", fused)):
        shard, _ = run(TPInfo(rank, world), comm, forced=full_toks)
        rows = torch.cat([rel_rows(a, b) for a, b in zip(full, shard)])
        err = rows.median().item()
        errs = [torch.zeros(2, device=dev) for _ in range(world)]
        dist.all_gather(errs, torch.tensor([err, rows.max().item()], device=dev))
        res[name] = [[round(v, 5) for v in e.tolist()] for e in errs]
    get_workspace(dev).check()
    # median row error at fp8 noise level on every rank (a routing near-tie may move one row)
    worst = max(e[0] for v in res.values() for e in v)
    ok = torch.tensor([1.0 if worst < 0.03 else 0.0], device=dev)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if rank == 0:
        print(json.dumps({"world": world, "ok": bool(ok.item() == 1.0),
                          "row_rel_err_median_max_per_rank": res}), flush=True)
    fused.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
