"""Tensor parallelism across GPUs: fused GEMM+all-reduce and NCCL paths vs. TP=1."""
import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_tp2_fused_and_nccl_match_tp1():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT)
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29531",
           "-m", "swarm_inference_lab_b200.parallel.selftest"]
    out = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT, timeout=400)
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert out.returncode == 0 and lines, out.stderr[-3000:]
    res = json.loads(lines[-1])
    assert res["ok"], res


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_mla_ep2_matches_ep1():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT)
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29533",
           "-m", "swarm_inference_lab_b200.parallel.ep_selftest"]
    out = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT, timeout=400)
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert out.returncode == 0 and lines, out.stderr[-3000:]
    res = json.loads(lines[-1])
    assert res["ok"], res
