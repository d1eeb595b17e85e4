"""Heterogeneous node roles and the measured utility harness (CPU): the role planner puts
nodes into the pipeline until the model fits, then makes replicas of nodes that can hold the
model, expert hosts of nodes that help an MoE, and leaves a node idle when it adds nothing;
the harness's background lane catches every tampered claim, its hybrid CPU-expert placement is
exact, and its evidence passes the frozen contract."""
import pytest

from swarm_inference_lab_b200.planner.roles import NodeCaps, assign_roles

GB = 1e9


def _roles(nodes, model_gb, **kw):
    return {r.node_id: (r.role, r.gain_tok_s) for r in assign_roles(nodes, model_gb * GB, **kw)}


def test_pipeline_members_until_the_model_fits_then_replicas():
    r = _roles([NodeCaps("a", 100.0, 10 * GB, 0.1), NodeCaps("b", 80.0, 10 * GB, 0.1),
                NodeCaps("c", 60.0, 20 * GB, 0.1)], 15)
    # a alone cannot hold 15 GB: a and b form the pipeline at the slower member's rate
    assert r["a"] == ("stage", 0.0) and r["b"] == ("stage", 80.0)
    assert r["c"] == ("replica", 60.0)


def test_a_node_that_adds_nothing_stays_idle():
    r = _roles([NodeCaps("big", 100.0, 20 * GB, 0.1), NodeCaps("small", 50.0, 2 * GB, 0.1)], 15)
    assert r["small"] == ("idle", 0.0)
    r = _roles([NodeCaps("big", 100.0, 20 * GB, 0.1), NodeCaps("far", 50.0, 2 * GB, 500.0)], 15,
               expert_fraction=0.3)
    assert r["far"] == ("idle", 0.0)              # the link costs more than the experts give


def test_an_moe_helper_hosts_experts():
    r = _roles([NodeCaps("big", 100.0, 20 * GB, 0.1), NodeCaps("helper", 50.0, 2 * GB, 0.05)], 15,
               expert_fraction=0.3)
    role, gain = r["helper"]
    assert role == "expert" and gain == pytest.approx(0.3 * 100 / 1.05 - 100 * 0.05 / 100)


def test_harness_evidence_passes_its_contract():
    from swarm_inference_lab_b200.testing.acceptance import check_contract, load_contract
    from swarm_inference_lab_b200.testing.heterogeneous import markdown, run
    rep = run(seconds=1.5, tokens=8)
    res = check_contract(load_contract("heterogeneous_utility"), rep)
    assert res["ok"], [r for r in res["results"] if not r["ok"]]
    b, c = rep["background_lane"], rep["cpu_experts"]
    assert b["caught"] == b["tampered"] > 0
    assert c["placements"].get("local", 0) > 0 and c["placements"].get("whole_remote", 0) > 0
    roles = {x["role"] for x in rep["node_roles"]["nodes"]}
    assert "stage" in roles and "idle" in roles        # the 0.4x-memory node adds nothing
    assert "capacity-normalised efficiency" in markdown(rep)
