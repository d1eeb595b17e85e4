"""Row-parallel projection + all-reduce: fused kernel vs. GEMM + NCCL (device-timed).

    torchrun --nproc-per-node N -m swarm_inference_lab_b200.parallel.tp_bench

For the Llama-3-8B attention-output (K = 4096/N) and down (K = 14336/N)
projections at 1, 32 and 128 tokens, times ``h += allreduce(x @ W^T)`` with
(a) the fused GEMM+all-reduce kernel and (b) the tcgen05 GEMM followed by NCCL
all-reduce and an add.  CUDA events, 20 iterations after warm-up, max over
ranks.  Rank 0 prints one JSON line per case.
"""
from __future__ import annotations

import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    from ..ops import gemm
    from .comm import NcclComm
    from .fused_tp import FusedTPComm
    nccl = NcclComm()
    fused = FusedTPComm(nccl, dev, max_tokens=128, hidden=4096)

    def timed(fn, iters=20):
        for _ in range(5):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(iters):
            fn()
        e.record()
        torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e) / iters * 1e3], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for K_full, name in ((4096, "o_proj"), (14336, "down_proj")):
        K = K_full // world
        w = (torch.randn(4096, K, device=dev) * 0.02).bfloat16()
        for T in (1, 32, 128):
            x = torch.randn(T, K, device=dev).bfloat16()
            h = torch.zeros(T, 4096, device=dev, dtype=torch.bfloat16)
            tf = timed(lambda: fused.fused_gemm_allreduce_residual(x, w, h))

            def unfused():
                o = gemm.linear(x, w)
                dist.all_reduce(o)
                h.add_(o)
            tn = timed(unfused)
            tg = timed(lambda: gemm.linear(x, w))
            if rank == 0:
                print(json.dumps({"world": world, "proj": name, "tokens": T, "fused_us": round(tf, 2),
                                  "gemm_plus_nccl_us": round(tn, 2), "gemm_only_us": round(tg, 2)}),
                      flush=True)
    fused.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
