"""Communicator selection on hosts without NVLink multicast (2 gloo CPU ranks): the NVLS
all-reduce reports itself unavailable on every rank instead of failing or hanging."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from swarm_inference_lab_b200.parallel.comm import NcclComm
        from swarm_inference_lab_b200.parallel.nvls_tp import NvlsTPComm
        base = NcclComm()          # a thin wrapper over the default (here: gloo) group
        q.put((rank, NvlsTPComm.available(base, torch.device("cpu"))))
    finally:
        dist.destroy_process_group()


def test_nvls_unavailable_without_multicast():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs)
    res = dict(q.get(timeout=5) for _ in range(2))
    assert res == {0: False, 1: False}
