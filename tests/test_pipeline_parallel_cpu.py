"""Micro-batched pipeline parallelism over gloo (2 CPU ranks) vs. a single process."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from swarm_inference_lab_b200.models.config import TINY_LLAMA_CPU
from swarm_inference_lab_b200.models.reference import ReferenceDecoder, random_source
from swarm_inference_lab_b200.parallel.pipeline import PipeGroup, PipelineStage

PROMPTS = [torch.randint(0, 32000, (n,), generator=torch.Generator().manual_seed(n)).tolist()
           for n in (12, 20, 7)]
STEPS = 4


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.set_num_threads(2)
    cfg = TINY_LLAMA_CPU
    per = cfg.num_layers // world
    model = ReferenceDecoder(cfg, random_source(0), layer_range=(rank * per, (rank + 1) * per))
    caches = [model.new_cache() for _ in PROMPTS]

    def fn(m, x):
        y = model.forward(x, caches[m])
        if model.with_head:
            return torch.argmax(y[-1:], dim=-1).to(torch.int64)
        return y.to(torch.float32)

    stage = PipelineStage(PipeGroup(rank, world, list(range(world))), fn, cfg.hidden_size,
                          dtype=torch.float32)
    stage.result_shape = lambda n: (1,)
    outs = [[] for _ in PROMPTS]
    # prefill (micro-batch m = one prompt), then decode steps fed by the returned tokens
    inputs = [torch.tensor(p) for p in PROMPTS] if rank == 0 else None
    res = stage.step(inputs, [len(p) for p in PROMPTS])
    for s in range(STEPS):
        if rank == 0:
            for m, r in enumerate(res):
                outs[m].append(int(r[0]))
            inputs = [r.clone() for r in res]
        res = stage.step(inputs, [1] * len(PROMPTS))
    if rank == 0:
        for m, r in enumerate(res):
            outs[m].append(int(r[0]))
        q.put(outs)
    dist.barrier()
    dist.destroy_process_group()


def test_pipeline_two_stages_match_single_process():
    torch.set_num_threads(2)
    ref = ReferenceDecoder(TINY_LLAMA_CPU, random_source(0))
    expect = [ref.greedy_generate(p, STEPS + 1)[0] for p in PROMPTS]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got == expect
