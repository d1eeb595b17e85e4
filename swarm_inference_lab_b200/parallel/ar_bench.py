"""All-reduce latency for decode-sized tensor-parallel sums: NCCL against the one-shot
NVLink kernels (device-timed, CUDA graph, max over ranks).

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m swarm_inference_lab_b200.parallel.ar_bench \
        [--hidden 4096] [--tokens 1,32,128] [--iters 64]

Per token count, each path runs ``--iters`` back-to-back all-reduces of a [tokens, hidden]
bf16 tensor inside one CUDA graph (the graph a decode step replays): ``nccl`` is
``dist.all_reduce`` in place; ``oneshot`` is ``oneshot_allreduce`` of a partial already in
the symmetric buffer into the residual stream; ``oneshot_norm`` also writes the next
block's RMSNorm input; ``ll`` / ``ll_norm`` are the low-latency kernel whose flag
travels inside each 8-byte word.  Rank 0 prints one JSON line per (path, tokens) with microseconds
per all-reduce and the NVLink roofline of a one-shot push (each rank sends its tensor to
every peer: (N-1) x bytes at the measured 770 GB/s per direction).
"""
from __future__ import annotations

import argparse
import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist

NVLINK_GBS = 770.0


def _graph_us(fn, iters: int, dev) -> float:
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for _ in range(3):
            fn()
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for _ in range(iters):
            fn()
    g.replay()
    torch.cuda.synchronize(dev)
    dist.barrier()
    best = float("inf")
    for _ in range(3):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        best = min(best, e0.elapsed_time(e1) * 1e3 / iters)
    t = torch.tensor([best], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    del g
    torch.cuda.synchronize(dev)
    dist.barrier()
    return float(t.item())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--tokens", default="1,32,128")
    ap.add_argument("--iters", type=int, default=64)
    a = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    from ..ops._ext import ext
    from ..ops.workspace import get_workspace
    from .comm import NcclComm
    from .ll_tp import LLTPComm
    from .oneshot_tp import OneShotTPComm
    toks = [int(t) for t in a.tokens.split(",")]
    H = a.hidden
    nccl = NcclComm()
    one = OneShotTPComm(nccl, dev, max_tokens=max(toks), hidden=H)
    ll = LLTPComm(nccl, dev, max_tokens=max(toks), hidden=H)
    st = get_workspace(dev).status
    nv = None
    if world > 1:
        from .nvls_tp import NvlsTPComm
        if NvlsTPComm.available(nccl, dev):
            nv = NvlsTPComm(nccl, dev, max_tokens=max(toks), hidden=H)
    nw = torch.ones(H, device=dev, dtype=torch.bfloat16)
    out = []
    for T in toks:
        g = torch.Generator(device=dev).manual_seed(rank * 1000 + T)
        part = one._partial(T, H)
        part.copy_(torch.randn(T, H, device=dev, generator=g).bfloat16())
        h = torch.zeros(T, H, device=dev, dtype=torch.bfloat16)
        x = torch.empty_like(h)
        buf = part.clone()

        def f_nccl():
            dist.all_reduce(buf)

        def f_one():
            ext().oneshot_allreduce(h, one.peers, one.rank, one.flags_off, one.recv_off,
                                    one.partial_off, one.max_elems, st)

        def f_norm():
            ext().oneshot_allreduce_norm(h, one.peers, one.rank, one.flags_off, one.recv_off,
                                         one.partial_off, one.max_elems, nw, 1e-5, x, st)
        ll._partial(T, H).copy_(part)

        def f_ll(two=False):
            ext().ll_allreduce_norm(h, ll.peers, ll.rank, ll.ll_off, ll.partial_off, ll.max_elems,
                                    None, 0.0, None, st, two)

        def f_ll_norm(two=False):
            ext().ll_allreduce_norm(h, ll.peers, ll.rank, ll.ll_off, ll.partial_off, ll.max_elems,
                                    nw, 1e-5, x, st, two)
        paths = [("nccl", f_nccl), ("oneshot", f_one), ("oneshot_norm", f_norm), ("ll", f_ll),
                 ("ll_norm", f_ll_norm)]
        if world > 1 and (H // 8) % world == 0:
            paths += [("ll_twoshot", lambda: f_ll(True)), ("ll_twoshot_norm", lambda: f_ll_norm(True))]
        if nv is not None:
            nv._partial(T, H).copy_(part)
            paths += [("nvls", lambda: nv._reduce(h)), ("nvls_norm", lambda: nv._reduce(h, nw, 1e-5, x))]
        bytes_ = T * H * 2
        roof_us = (world - 1) * bytes_ / (NVLINK_GBS * 1e3)
        for name, fn in paths:
            us = _graph_us(fn, a.iters, dev)
            out.append({"path": name, "world": world, "tokens": T, "hidden": H, "bytes": bytes_,
                        "us_per_allreduce": round(us, 2), "nvlink_roofline_us": round(roof_us, 2)})
    get_workspace(dev).check()
    if rank == 0:
        print(json.dumps({"nvls_multicast": nv is not None}), flush=True)
        for r in out:
            print(json.dumps(r), flush=True)
    # Correctness of the NVLS sum against NCCL on the last token count.
    if nv is not None:
        T = toks[-1]
        g = torch.Generator(device=dev).manual_seed(rank + 7)
        p = torch.randn(T, H, device=dev, generator=g).bfloat16()
        nv._partial(T, H).copy_(p)
        hh = torch.zeros(T, H, device=dev, dtype=torch.bfloat16)
        nv._reduce(hh)
        ref = p.float()
        dist.all_reduce(ref)
        err = (hh.float() - ref).abs().max().item()
        if rank == 0:
            print(json.dumps({"nvls_check_max_abs_err": err, "ref_max": ref.abs().max().item()}), flush=True)
        nv.close()
    one.close()
    ll.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
