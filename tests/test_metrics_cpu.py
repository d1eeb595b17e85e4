"""Process metrics (counters, gauges, latency summaries; JSON and Prometheus text) and the
JSON log formatter."""
import io
import json
import logging

from swarm_inference_lab_b200.telemetry.metrics import JsonLogFormatter, Metrics


def test_metrics_snapshot_and_prometheus():
    m = Metrics(window=8)
    m.inc("requests")
    m.inc("requests", 2)
    m.inc("frames", stage=1, op="DECODE")
    m.set("workers_healthy", 3)
    for v in range(1, 11):
        m.observe("tpot_ms", float(v))
    snap = m.snapshot()
    assert snap["counters"]["requests"] == 3
    assert snap["counters"]['frames{op="DECODE",stage="1"}'] == 1
    assert snap["gauges"]["workers_healthy"] == 3
    s = snap["summaries"]["tpot_ms"]
    assert s["count"] == 10 and s["sum"] == 55.0 and s["p50"] in (6.0, 7.0)  # window of 8
    text = m.prometheus()
    assert "swarm_requests_total 3" in text
    assert 'swarm_frames_total{op="DECODE",stage="1"} 1' in text
    assert "swarm_tpot_ms_count 10" in text
    assert 'swarm_tpot_ms{quantile="0.99"}' in text


def test_json_log_formatter():
    buf = io.StringIO()
    h = logging.StreamHandler(buf)
    h.setFormatter(JsonLogFormatter())
    log = logging.getLogger("swarm.test.json")
    log.addHandler(h)
    log.setLevel(logging.INFO)
    log.info("stage %d ready", 3, extra={"worker": "n1", "generation": 7})
    rec = json.loads(buf.getvalue().strip())
    assert rec["msg"] == "stage 3 ready" and rec["level"] == "INFO"
    assert rec["worker"] == "n1" and rec["generation"] == 7
    log.removeHandler(h)
