"""Intra-box link probe: NVLink peer-copy bandwidth/latency and all-reduce cost, fitted
into the constants the box planner uses (``planner/box_planner.BoxMeasurements``).

    torchrun --nproc-per-node N -m swarm_inference_lab_b200.parallel.nvlink_probe --out probe.json

Rank 0 times device-to-device copies to every peer (CUDA events on the
source stream, 256 MiB for bandwidth, 4 KiB for latency); all ranks then
time NCCL all-reduces from 8 KiB to 64 MiB (max over ranks) and fit
``alpha + beta * MB``.  The result also yields directed ``LinkProfile``s of
the ``nvlink`` domain for the topology layer.

Reference: the directed network measurement of si/cluster/network.py:395-620,
extended to the GPU-to-GPU domain.
"""
from __future__ import annotations

import argparse
import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist


def _time(fn, iters=10):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def peer_copy(src: int, dst: int, nbytes: int) -> float:
    a = torch.empty(nbytes, dtype=torch.uint8, device=f"cuda:{src}")
    b = torch.empty(nbytes, dtype=torch.uint8, device=f"cuda:{dst}")
    with torch.cuda.device(src):
        return _time(lambda: b.copy_(a, non_blocking=True))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default="nvlink_probe.json")
    a = ap.parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    res = {"world": world, "links": []}
    if rank == 0 and torch.cuda.device_count() > 1:
        bws, lats = [], []
        for d in range(1, torch.cuda.device_count()):
            ms = peer_copy(0, d, 256 << 20)
            lat = peer_copy(0, d, 4096) * 1e3
            bw = (256 << 20) / (ms / 1e3) / 1e9
            bws.append(bw)
            lats.append(lat)
            res["links"].append({"src": "cuda:0", "dst": f"cuda:{d}", "gbs": bw, "latency_us": lat})
        res["nvlink_gbs"] = sorted(bws)[len(bws) // 2]
        res["nvlink_latency_us"] = sorted(lats)[len(lats) // 2]
    if world > 1:
        samples = []
        for size in (8 << 10, 64 << 10, 256 << 10, 1 << 20, 4 << 20, 16 << 20, 64 << 20):
            x = torch.ones(size // 2, dtype=torch.bfloat16, device="cuda")
            ms = _time(lambda: dist.all_reduce(x), iters=20)
            t = torch.tensor([ms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            samples.append((size, float(t.item()) * 1e3))
        res["allreduce_samples_us"] = samples
        from ..planner.box_planner import BoxMeasurements
        m = BoxMeasurements()
        m.fit_allreduce(samples[:4])
        res["ar_alpha_us"] = m.ar_alpha_us
        res["ar_beta_us_per_mb"] = m.ar_beta_us_per_mb
        big = samples[-1]
        res["allreduce_busbw_gbs"] = 2 * (world - 1) / world * big[0] / (big[1] / 1e6) / 1e9
    if rank == 0:
        with open(a.out, "w") as f:
            json.dump(res, f, indent=1)
        print(json.dumps(res))
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
