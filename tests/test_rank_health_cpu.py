"""Host-side rank failure detection (CPU, gloo, 3 ranks as processes): a rank that dies
silently between steps, one that raises, one that leaves in order, and one that never joins
are all reported -- by name and reason -- to the surviving ranks at their next step, before or
instead of a hung collective."""
import multiprocessing as mp
import os
import socket
import traceback
from datetime import timedelta

import pytest


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(scenario, rank, world, port, q):
    import torch
    import torch.distributed as dist

    from swarm_inference_lab_b200.parallel.rank_health import RankFailure, RankMonitor
    store = dist.TCPStore("127.0.0.1", port, world_size=None, is_master=(rank == 0),
                          timeout=timedelta(seconds=30), wait_for_workers=False)
    mon = None
    try:
        mon = RankMonitor("127.0.0.1", port, rank, world, interval_s=0.1, timeout_s=1.0)
        mon.start(join_timeout_s=3.0)
        dist.init_process_group("gloo", store=store, rank=rank, world_size=world,
                                timeout=timedelta(seconds=5))
        t = torch.ones(4)
        for step in range(8):
            mon.check()
            if scenario == "raise" and rank == 1 and step == 2:
                raise ValueError("boom at step 2")
            with mon.guard():
                dist.all_reduce(t)
            if step == 3 and rank == 2:
                if scenario == "silent":
                    os._exit(0)                       # no announcement, no heartbeat
                if scenario == "leave":
                    mon.leave()
                    q.put((rank, "left", None))
                    return
        q.put((rank, "finished", None))
    except RankFailure as f:
        q.put((rank, "failure", f.ranks))
    except Exception as exc:  # noqa: BLE001 - the reason goes to the others and the test
        if mon is not None:
            mon.fail(f"{type(exc).__name__}: {exc}")
        q.put((rank, "raised", f"{type(exc).__name__}: {exc}"))
        if scenario == "raise":
            q.close()
            q.join_thread()                           # flush the report before dying
            os._exit(1)
        q.put((rank, "trace", traceback.format_exc()))
    finally:
        if mon is not None:
            mon.stop()
        if rank == 0:
            import time
            time.sleep(1.5)                           # keep the store up for the others


def _run(scenario, ranks=(0, 1, 2), world=3):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(scenario, r, world, port, q)) for r in ranks]
    for p in procs:
        p.start()
    out = {}
    try:
        for p in procs:
            p.join(timeout=90)
        while not q.empty():
            r, kind, detail = q.get()
            out.setdefault(r, []).append((kind, detail))
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()
                p.join(timeout=10)
    return out


@pytest.mark.timeout(180)
def test_a_silent_death_is_named_by_the_survivors():
    out = _run("silent")
    for r in (0, 1):
        (kind, ranks), = [e for e in out[r] if e[0] != "trace"]
        assert kind == "failure" and list(ranks) == [2] and "silent" in ranks[2], out


@pytest.mark.timeout(180)
def test_a_raising_rank_reports_its_reason():
    out = _run("raise")
    assert out[1][0] == ("raised", "ValueError: boom at step 2")
    for r in (0, 2):
        (kind, ranks), = [e for e in out[r] if e[0] != "trace"]
        assert kind == "failure" and ranks == {1: "failed: ValueError: boom at step 2"}, out


@pytest.mark.timeout(180)
def test_an_orderly_leave_stops_the_others_before_their_next_collective():
    out = _run("leave")
    assert out[2] == [("left", None)]
    for r in (0, 1):
        assert out[r] == [("failure", {2: "left"})], out


@pytest.mark.timeout(180)
def test_a_rank_that_never_joins_is_reported():
    out = _run("never", ranks=(0, 1), world=3)
    for r in (0, 1):
        assert out[r] == [("failure", {2: "never joined"})], out


def _pipe_rank(rank, world, port, q):
    import torch
    import torch.distributed as dist

    from swarm_inference_lab_b200.parallel.pipeline import PipeGroup, PipelineStage
    from swarm_inference_lab_b200.parallel.rank_health import RankFailure, RankMonitor
    store = dist.TCPStore("127.0.0.1", port, world_size=None, is_master=(rank == 0),
                          timeout=timedelta(seconds=30), wait_for_workers=False)
    mon = RankMonitor("127.0.0.1", port, rank, world, interval_s=0.1, timeout_s=1.0).start(3.0)
    dist.init_process_group("gloo", store=store, rank=rank, world_size=world,
                            timeout=timedelta(seconds=5))
    H = 8

    def fn(m, x):
        if rank == 0:
            return torch.ones(x.shape[0], H) * x.float().sum()
        return x.sum(dim=0, keepdim=True)[:, :1].to(torch.int64)

    stage = PipelineStage(PipeGroup(rank, world, list(range(world))), fn, H, dtype=torch.float32,
                          monitor=mon)
    stage.result_shape = lambda n: (1, 1)
    try:
        for step in range(6):
            stage.step([torch.tensor([1, 2, 3])] if rank == 0 else None, [3])
            if rank == 1 and step == 1:
                os._exit(0)                           # the last stage dies between steps
        q.put((rank, "finished", None))
    except RankFailure as f:
        q.put((rank, "failure", f.ranks))
    finally:
        mon.stop()
        import time
        time.sleep(1.0)


@pytest.mark.timeout(180)
def test_pipeline_stage_names_a_dead_next_stage():
    """A 2-stage gloo pipeline with a monitor: when the last stage dies between steps, the
    first stage's next step ends with ``RankFailure`` naming it instead of hanging."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_pipe_rank, args=(r, 2, port, q)) for r in (0, 1)]
    for p in procs:
        p.start()
    try:
        for p in procs:
            p.join(timeout=90)
        got = [q.get(timeout=10)]
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()
                p.join(timeout=10)
    (rank, kind, ranks), = got
    assert rank == 0 and kind == "failure" and list(ranks) == [1] and "silent" in ranks[1]
