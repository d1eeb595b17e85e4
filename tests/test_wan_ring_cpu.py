"""Stage-ring decode over emulated network profiles (CPU): a 2-stage tiny-Llama ring with a
delaying proxy on each hop produces the single-process greedy tokens at every profile, with
two request messages and two serial waits per decoded token, per-token latency above the
emulated network floor, and the ``stage_ring_wan`` contract passing; a session close reaches
every stage."""
import asyncio

import torch


def test_wan_ring_profiles_meet_the_contract():
    from swarm_inference_lab_b200.testing.acceptance import check_contract, load_contract
    from swarm_inference_lab_b200.testing.wan_ring import evidence, run
    torch.set_num_threads(2)
    rows = asyncio.run(run(["loopback", "wifi"], tokens=5))
    for r in rows:
        assert r["exact_tokens"], r
        assert r["messages_per_token"] == 2.0, r
        assert r["stage_sessions_closed"] == [1, 1], r
        assert r["stage_errors"] == [0, 0], r
    wifi = rows[1]
    assert wifi["ms_per_token"] >= wifi["network_floor_ms"], wifi
    rep = check_contract(load_contract("stage_ring_wan"), evidence(rows))
    assert rep["ok"], rep


def test_strategy_planner_keeps_only_faster_exact_options():
    from swarm_inference_lab_b200.testing.wan_ring import plan_strategy
    torch.set_num_threads(2)
    d = asyncio.run(plan_strategy("wifi", tokens=8))
    scores = {x["candidate"]: x for x in d["scores"]}
    assert set(scores) == {"plain", "compressed", "speculative"}
    assert all(x["feasible"] for x in scores.values())          # every candidate is exact
    best = min(scores.values(), key=lambda x: x["ms_per_token"])
    assert d["selected"] == best["candidate"] and scores[d["selected"]]["selected"]
    assert scores["speculative"]["serial_waits_per_token"] < scores["plain"]["serial_waits_per_token"]
