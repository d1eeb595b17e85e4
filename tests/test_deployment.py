"""Deployment manager phases, rollback and recovery with in-process worker agents (CPU)."""
import asyncio

import pytest

from swarm_inference_lab_b200.coordinator.deployment import (DeploymentError, DeploymentManager, LoadReport,
                                                             Phase, StagePlan)
from swarm_inference_lab_b200.coordinator.state import DurableState, WorkerRecord, WorkerRegistry
from swarm_inference_lab_b200.security.identity import Identity, LeaseVerifier


class FakeAgent:
    def __init__(self, wid, artifacts, *, fail=None, free=1 << 40):
        self.worker_id = wid
        self.ident = Identity.generate(wid)
        self.fingerprint = self.ident.fingerprint
        self.endpoint = f"127.0.0.1:{9000 + int(wid[1:])}"
        self.artifacts = set(artifacts)
        self.fail = fail or set()
        self.free = free
        self.reserved = None
        self.loaded = None
        self.routes = []
        self.verifier = None

    async def reserve(self, dep, stage):
        self.reserved = dep
        return "reserve" not in self.fail

    async def release(self, dep):
        self.reserved = None

    async def has_artifact(self, aid):
        return aid in self.artifacts

    async def fetch_artifact(self, aid):
        if "fetch" in self.fail:
            raise IOError("transfer interrupted")
        self.artifacts.add(aid)

    async def verify_artifact(self, aid):
        return aid in self.artifacts and "verify" not in self.fail

    async def load_stage(self, plan):
        if "load" in self.fail:
            raise RuntimeError("out of memory")
        self.loaded = plan
        return LoadReport(plan.artifact_id, 10, plan.artifact_bytes)

    async def unload_stage(self, dep):
        self.loaded = None

    async def install_route(self, signed, nxt):
        lease = self.verifier.verify(signed, worker_fingerprint=self.fingerprint)
        self.routes.append((lease.generation, nxt))

    async def withdraw_route(self, gen):
        self.routes = [r for r in self.routes if r[0] != gen]

    async def check_peer(self, ep):
        return "peer" not in self.fail

    async def free_bytes(self):
        return self.free


def _setup(tmp_path, fails=None, n=3):
    coord = Identity.generate("coordinator")
    reg = WorkerRegistry()
    agents = {}
    for i in range(n):
        wid = f"w{i}"
        a = FakeAgent(wid, {"A0"} if i == 0 else set(), fail=(fails or {}).get(wid))
        a.verifier = LeaseVerifier(coord.fingerprint)
        agents[wid] = a
        reg.register(WorkerRecord(wid, a.fingerprint, a.endpoint))
    mgr = DeploymentManager(reg, agents, coord, DurableState(tmp_path / "state.json"))
    plan = [StagePlan(0, "w0", 0, 2, "A0", 100), StagePlan(1, "w1", 2, 4, "A1", 100)]
    return mgr, agents, plan


def test_deploy_ready_with_transfer_and_signed_routes(tmp_path):
    mgr, agents, plan = _setup(tmp_path)
    d = asyncio.run(mgr.deploy(plan, model_revision="rev", topology_id="t"))
    phases = [p for p, _ in d.history]
    assert phases == ["RESERVING", "PREPARING", "TRANSFERRING", "VERIFYING_ARTIFACTS", "LOADING",
                      "VERIFYING_LOADS", "INSTALLING_ROUTES", "VERIFYING_PEERS", "READY"]
    assert agents["w1"].artifacts == {"A1"}
    assert agents["w0"].routes == [(d.generation, agents["w1"].endpoint)]
    assert agents["w1"].routes == [(d.generation, None)]


@pytest.mark.parametrize("where", ["fetch", "load", "peer", "reserve"])
def test_failure_rolls_back(tmp_path, where):
    mgr, agents, plan = _setup(tmp_path, {"w0" if where == "peer" else "w1": {where}})
    with pytest.raises(DeploymentError):
        asyncio.run(mgr.deploy(plan, model_revision="rev", topology_id="t"))
    d = next(iter(mgr.deployments.values()))
    assert d.phase == Phase.FAILED and d.error
    for a in agents.values():
        assert a.loaded is None and a.reserved is None and a.routes == []


def test_recover_replaces_worker_and_fences_old_generation(tmp_path):
    mgr, agents, plan = _setup(tmp_path)
    d = asyncio.run(mgr.deploy(plan, model_revision="rev", topology_id="t"))
    g0 = d.generation
    d = asyncio.run(mgr.recover(d.deployment_id, "w1"))
    assert d.phase == Phase.READY and d.generation > g0
    assert [s.worker_id for s in d.stages] == ["w0", "w2"]
    assert agents["w0"].routes[-1] == (d.generation, agents["w2"].endpoint)
    # a replayed old lease is rejected by the stage's verifier (generation fence)
    with pytest.raises(Exception):
        asyncio.run(agents["w0"].install_route(mgr._lease(type(d)(d.deployment_id, "rev", "t", d.stages,
                                                                   generation=g0)), None))


def test_recover_without_candidates_fails(tmp_path):
    mgr, agents, plan = _setup(tmp_path, n=2)
    d = asyncio.run(mgr.deploy(plan, model_revision="rev", topology_id="t"))
    with pytest.raises(DeploymentError, match="no eligible replacement"):
        asyncio.run(mgr.recover(d.deployment_id, "w1"))


def test_unload(tmp_path):
    mgr, agents, plan = _setup(tmp_path)
    d = asyncio.run(mgr.deploy(plan, model_revision="rev", topology_id="t"))
    asyncio.run(mgr.unload(d.deployment_id))
    assert d.phase == Phase.UNLOADED
    assert all(a.loaded is None and a.routes == [] for a in agents.values())
