"""Integrity audits, replay log, stage sessions, residency, engine processes, canonical facade (CPU)."""
import json
import sys

import pytest
import torch

from swarm_inference_lab_b200.coordinator.integrity import IntegrityCoordinator, ReputationBook
from swarm_inference_lab_b200.coordinator.replay_log import ReplayLog, ReplayLogError
from swarm_inference_lab_b200.runtime.processes import (EngineProcess, ProcessVerificationError, file_digest,
                                                        shutdown_all)
from swarm_inference_lab_b200.runtime.residency import ResidencyTracker
from swarm_inference_lab_b200.runtime.sessions import StageSessionRegistry


def test_integrity_quarantines_the_disagreeing_worker():
    ic = IntegrityCoordinator(ReputationBook(max_mismatches=2))
    a = torch.arange(10)
    assert ic.judge("w0", a, "w1", a.clone())
    for _ in range(2):
        assert not ic.judge("w2", a + 1, "w1", a, tiebreak=("w0", a.clone()))
    assert not ic.book.eligible("w2") and ic.book.eligible("w1")
    assert ic.judge("w0", torch.ones(3), "w1", torch.ones(3) + 1e-5, exact=False)


def test_replay_log_roundtrip_and_tamper_detection(tmp_path):
    log = ReplayLog(tmp_path)
    log.open("r1", [5, 6, 7])
    log.accept("r1", 3, 11)
    log.accept("r1", 4, 12)
    with pytest.raises(ReplayLogError):
        log.accept("r1", 9, 13)
    log.finish("r1")
    assert log.replay_inputs("r1") == [5, 6, 7, 11, 12]
    rec = ReplayLog(tmp_path).load("r1")
    assert rec.tokens == [11, 12] and rec.state == "finished"
    p = tmp_path / "r1.jsonl"
    p.write_text(p.read_text().replace("[3, 11]", "[3, 99]"))
    with pytest.raises(ReplayLogError, match="chain"):
        ReplayLog(tmp_path).load("r1")


def test_stage_sessions_generation_fence_ttl_and_lru():
    reg = StageSessionRegistry(max_sessions=2, idle_ttl_s=10)
    evicted = []
    reg.open("a", "t", 1, now=0)
    reg.open("b", "t", 1, now=1)
    reg.get("a", topology_id="t", generation=1, now=2)
    reg.open("c", "t", 2, now=3, evict=evicted.append)        # LRU evicts b
    assert [s.session_id for s in evicted] == ["b"]
    with pytest.raises(KeyError):
        reg.get("a", topology_id="t", generation=2)
    reg.advance("a", 5)
    with pytest.raises(ValueError):
        reg.advance("a", 4)
    assert reg.invalidate_generation(2) == ["a"]
    assert reg.expire(now=100) == ["c"]


def test_residency_tracker():
    rt = ResidencyTracker()
    rt.place("e0", "device:0", 100)
    rt.place("e1", "host_pinned", 50)
    rt.place("emb", "device:0", 10, pinned=True)
    assert rt.lookup("e0", "device:0") and not rt.lookup("e1", "device:0")
    rt.move("e1", "device:0", 0.001)
    assert rt.bytes_on() == {"device:0": 160}
    assert rt.moved_bytes(dst="device:0") == 50
    with pytest.raises(ValueError):
        rt.move("emb", "host")
    assert rt.evict_candidates("device:0", 60) == ["e0"]


def test_engine_process_verify_start_stop(tmp_path):
    script = tmp_path / "w.py"
    script.write_text("import json,time,sys\nprint(json.dumps({'ready': True, 'port': 1}), flush=True)\n"
                      "time.sleep(60)\n")
    p = EngineProcess([sys.executable, str(script)], verify={str(script): file_digest(script)})
    assert p.start(ready_timeout_s=30)["port"] == 1
    assert p.alive()
    assert shutdown_all([p], 10) == ["terminated"]
    bad = EngineProcess([sys.executable, str(script)], verify={str(script): "0" * 64})
    with pytest.raises(ProcessVerificationError):
        bad.start()


def test_canonical_runtime_dry_run():
    from swarm_inference_lab_b200.engines import ClusterCapabilities, RequestShape
    from swarm_inference_lab_b200.runtime.canonical import CanonicalRuntime
    rt = CanonicalRuntime()
    info = rt.inspect("kimi-k2-shape")
    assert info["mla"] and info["parameters"] > 9e11
    caps = ClusterCapabilities(nodes={"local": {"gpus": 8, "gpu_name": "NVIDIA B200"}})
    r = rt.dry_run("llama-3-8b-shape", caps, RequestShape(batch=32, prompt_tokens=2048,
                                                           output_tokens=256, mode="throughput"))
    assert r["winner"]["engine"] == "native-stage"
    json.dumps(r)
