"""The loopback replica-scaling harness on the real control plane (tiny fp32 Llama, CPU):
every request is verified against the single-process tokens, both replicas serve, and the
fan-out timings (acquisition, cold and warm deploy) are reported."""
import asyncio

from swarm_inference_lab_b200.testing.loopback_matrix import markdown, run_matrix


def test_loopback_matrix_two_workers():
    rows = asyncio.run(run_matrix([2], [1, 4], stages=1, tokens=6))
    assert len(rows) == 2
    for r in rows:
        assert r["verified_requests"] == r["concurrency"]
        assert r["verified_tokens_per_s"] > 0
        assert r["cold_deploy_ms"] > 0 and r["warm_deploy_ms"] > 0 and r["acquire_ms"] > 0
    assert set(rows[1]["requests_per_replica"]) == {"replica0", "replica1"}
    assert "| 2 | 2 | 4 |" in markdown(rows)
