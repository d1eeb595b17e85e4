"""Frozen acceptance contracts: the checker passes a conforming evidence record (the
headline bench line) and names the failing gate of a non-conforming one."""
import copy
import json

from swarm_inference_lab_b200.testing.acceptance import check_contract, load_contract, main

GOOD = {"metric": "decode tokens/s/box + p50 TTFT/TPOT, K2-shape fp8 EP & 8B TP at 1/2/4/8 GPU",
        "value": 6508.1, "unit": "tokens/s", "dtype": "bf16", "steps": 64, "warmup": 3,
        "config": {"model": "llama-3-8b-shape", "global_batch": 32, "seq_len": 2048},
        "e2e": {"value": 6357.3, "h2d_bytes_per_step": 5504}, "gpu_launches": 16640,
        "clocks": {"reasons": []}, "ttft_ms_p50": 1239.5}


def test_headline_contract_passes_and_fails(tmp_path):
    c = load_contract("dense_decode_8b")
    assert check_contract(c, GOOD)["ok"]
    bad = copy.deepcopy(GOOD)
    bad["warmup"] = 1
    bad["clocks"]["reasons"] = ["hw_thermal_slowdown"]
    rep = check_contract(c, bad)
    failed = {r["field"] for r in rep["results"] if not r["ok"]}
    assert failed == {"warmup", "clocks.reasons"}
    p = tmp_path / "bench.log"
    p.write_text("noise\n" + json.dumps(GOOD) + "\n")
    assert main(["dense_decode_8b", str(p)]) == 0


def test_every_shipped_contract_loads():
    from pathlib import Path

    from swarm_inference_lab_b200.testing.acceptance import CONTRACTS
    names = {p.stem for p in Path(CONTRACTS).glob("*.yaml")}
    assert {"dense_decode_8b", "cpu_plumbing", "tp_exactness", "promotion_manifest",
            "stage_ring_wan", "real_loopback", "heterogeneous_utility"} <= names
    for name in names:
        assert load_contract(name)["contract_version"] == 1
    listed = set(load_contract("promotion_manifest")["contracts"])
    assert listed <= names
