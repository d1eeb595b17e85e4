"""Evidence bundles (``testing/reporting.py``, CLI ``report``): scaling figures from bench
lines at several GPU counts, CSV per record kind, a self-contained HTML page with inline SVG
charts, and a summary whose status fails on a failed contract or exactness check."""
import json

import pytest

from swarm_inference_lab_b200.testing import reporting


def _bench(n, v, impl="ours"):
    return {"metric": "decode_tokens_per_s", "value": v, "unit": "tokens/s", "n_gpus": n,
            "ms_per_step": 32 / v * 1e3, "impl": impl, "dtype": "bf16",
            "config": {"model": "llama-3-8b-shape", "parallelism": f"tp{n}"},
            "clocks": {"sm_mhz": 1965.0}}


WAN = {"name": "stage_ring_wan", "rows": [
    {"profile": p, "one_way_ms": ow, "exact_tokens": True, "ms_per_token": ms,
     "network_floor_ms": 2 * ow, "decode_tokens_per_s": 1e3 / ms, "messages_per_token": 2.0,
     "payload_bytes_per_token": 5400, "serial_waits_per_token": 2.0}
    for p, ow, ms in (("loopback", 0, 3.0), ("wifi", 4, 12.0), ("global", 75, 160.0))]}
LOOP = [{"workers": w, "replicas": w, "concurrency": c, "verified_tokens_per_s": 100.0 * w * min(c, w),
         "verified_requests": c, "latency_ms_p50": 10.0, "latency_ms_p99": 20.0,
         "cold_deploy_ms": 300.0, "warm_deploy_ms": 30.0} for w in (2, 4) for c in (1, 16)]
REAL = {"checkpoint": "/ck", "family": "qwen3", "stages": [{"layers": [0, 2], "worker": "a"},
                                                        {"layers": [2, 4], "worker": "b"}],
        "prompt": [1, 2], "tokens": [5, 6, 7], "reference_tokens": [5, 6, 7],
        "reference": "transformers generate (fp32)", "exact": True, "seconds": 40.0}
EXPERT = [{"backend": b, "tokens": 8, "ms_per_forward": ms, "expert_requests": r,
           "remote_rows_served": rows, "max_abs_logit_diff": 0.0, "exact": True}
          for b, ms, r, rows in (("local", 5.0, 0, 0), ("microshard_2", 20.0, 32, 64))]


def test_scaling_rows_gain_efficiency_and_marginal():
    rows = reporting.scaling_rows([_bench(1, 6500.0), _bench(2, 9100.0), _bench(4, 11700.0),
                                   _bench(8, 13000.0), _bench(1, 500.0, "reference")])
    assert [r["n_gpus"] for r in rows] == [1, 2, 4, 8]          # one N only: no reference rows
    by_n = {r["n_gpus"]: r for r in rows}
    assert by_n[1]["gain"] == 1.0 and by_n[1]["efficiency"] == 1.0
    assert by_n[2]["gain"] == pytest.approx(1.4) and by_n[2]["efficiency"] == pytest.approx(0.7)
    assert by_n[4]["marginal_per_gpu"] == pytest.approx((11700 - 9100) / 2)
    assert by_n[8]["efficiency"] == pytest.approx(13000 / 6500 / 8)
    assert reporting.capacity_efficiency(90.0, [100.0, 120.0, 150.0]) == pytest.approx(0.9)
    assert reporting.capacity_efficiency(90.0, []) == 0.0


def test_kinds_and_csv():
    recs = [_bench(1, 6500.0), WAN, REAL, *LOOP, *EXPERT, {"something": {"nested": 1}}]
    assert [reporting.kind(r) for r in recs[:3]] == ["bench", "wan", "real_loopback"]
    rows = reporting.rows_by_kind(recs)
    assert len(rows["wan"]) == 3 and len(rows["loopback"]) == 4 and len(rows["expert_backend"]) == 2
    assert rows["other"][0] == {"something.nested": 1}
    text = reporting.to_csv(rows["bench"])
    head, line = text.splitlines()[:2]
    assert "config.parallelism" in head.split(",") and "clocks.sm_mhz" in head.split(",")
    assert line.split(",")[head.split(",").index("value")] == "6500.0"


def test_bundle_html_and_status(tmp_path):
    from swarm_inference_lab_b200.testing.acceptance import check_contract, load_contract
    ok = check_contract(load_contract("stage_ring_wan"), {"exact_tokens": True})
    recs = [_bench(1, 6500.0), _bench(2, 9100.0), WAN, REAL, *LOOP, *EXPERT]
    s = reporting.write_bundle(recs, tmp_path / "b")
    assert s["status"] == "PASS" and s["exactness_checks"] == 3 + 1 + 2
    files = {p.name for p in (tmp_path / "b").iterdir()}
    assert {"report.html", "report.md", "summary.json", "records.jsonl", "bench.csv", "wan.csv",
            "loopback.csv", "scaling.csv", "real_loopback.csv", "expert_backend.csv"} <= files
    page = (tmp_path / "b" / "report.html").read_text()
    assert page.count("<svg") == 6      # bench bars, scaling x2, loopback lines, WAN, experts
    assert "Status: <span class='ok'>PASS</span>" in page
    # a failed contract and a non-exact row turn the status to FAIL
    bad = dict(REAL, exact=False)
    s = reporting.write_bundle([ok, bad], tmp_path / "c")
    assert s["status"] == "FAIL" and "exactness" in s["failed"]
    assert s["contracts_failed"] == (0 if ok["ok"] else 1)


def test_cli_report_bundle_and_formats(tmp_path):
    from typer.testing import CliRunner

    from swarm_inference_lab_b200.cli import app
    log = tmp_path / "scale.log"
    log.write_text("\n".join(json.dumps(_bench(n, v)) for n, v in ((1, 6500.0), (4, 11700.0))))
    ev = tmp_path / "expert.json"
    ev.write_text(json.dumps(EXPERT))
    run = CliRunner().invoke
    r = run(app, ["report", str(log), str(ev), "--out", str(tmp_path / "bundle")])
    assert r.exit_code == 0, r.output
    assert json.loads(r.output.strip().splitlines()[-1])["kinds"] == {"bench": 2, "expert_backend": 2}
    r = run(app, ["report", str(log), "--format", "md"])
    assert "| ours | llama-3-8b-shape | 4 | tp4 | 11700.0 tokens/s | 1.80 | 0.45 |" in r.output
    r = run(app, ["report", str(ev), "--format", "csv"])
    assert r.output.startswith("# expert_backend\nbackend,tokens,ms_per_forward")
    r = run(app, ["report", str(log), "--format", "html"])
    assert r.output.lstrip().startswith("<!doctype html>") and "<svg" in r.output
