"""A real checkpoint served as process-isolated pipeline stages on one host, checked token for
token against the model's own greedy generation.

    python -m swarm_inference_lab_b200.testing.real_loopback CHECKPOINT --stages 4 --tokens 24
    swarm experiment real-loopback CHECKPOINT --stages 4

Everything goes through the public commands, each node in its own OS process: ``swarm cluster
create`` + ``cluster start`` (coordinator process: pairing and the mutual-TLS control plane),
per node ``cluster pair`` -> ``node join`` -> ``node agent`` (registers, heartbeats, loads the
stage it is assigned from the checkpoint's safetensors), then ``swarm run CHECKPOINT
--require-distributed --stages N``.  The reference is the checkpoint's own greedy decode:
Hugging Face ``generate`` (fp32) when ``transformers`` is installed, else this repository's
fp32 reference decoder on the same weights.  Reported: per-stage layer intervals and workers,
the tokens, the reference tokens, exactness, and wall time.

Reference: si/experiments/experiment_002.py (real Qwen3 checkpoint, 4-stage process-isolated
exact-token validation) and the ``real-experiment`` command of si/cli.py.
"""
from __future__ import annotations

import argparse
import json
import os
import random
import signal
import socket
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

ROOT = str(Path(__file__).resolve().parents[2])


def _env() -> dict:
    return dict(os.environ, PYTHONPATH=ROOT, OMP_NUM_THREADS="2", CUDA_VISIBLE_DEVICES="")


def _swarm(*args, timeout=300):
    out = subprocess.run([sys.executable, "-m", "swarm_inference_lab_b200.cli", *args],
                         capture_output=True, text=True, env=_env(), cwd=ROOT, timeout=timeout)
    if out.returncode != 0:
        raise RuntimeError(f"swarm {' '.join(args)} failed:\n{out.stdout}\n{out.stderr[-3000:]}")
    return out.stdout


def _free_pair() -> int:
    for _ in range(200):
        p = random.randint(20000, 60000)
        ok = True
        for q in (p, p + 1):
            with socket.socket() as s:
                try:
                    s.bind(("127.0.0.1", q))
                except OSError:
                    ok = False
        if ok:
            return p
    raise RuntimeError("no free port pair")


def reference_tokens(checkpoint: str, prompt: list[int], tokens: int) -> tuple[list[int], str]:
    try:
        from transformers import AutoModelForCausalLM
        hf = AutoModelForCausalLM.from_pretrained(checkpoint, torch_dtype=torch.float32).eval()
        with torch.no_grad():
            out = hf.generate(torch.tensor([prompt]), max_new_tokens=tokens, do_sample=False)
        return out[0, len(prompt):].tolist(), "transformers generate (fp32)"
    except ImportError:
        from ..model_io.loader import checkpoint_config, safetensors_source
        from ..models.reference import ReferenceDecoder
        cfg = checkpoint_config(checkpoint)
        out = ReferenceDecoder(cfg, safetensors_source(checkpoint)).greedy_generate(prompt, tokens)[0]
        stop = next((i for i, t in enumerate(out) if t in cfg.eos_token_ids), None)
        return (out if stop is None else out[:stop + 1]), "reference decoder (fp32)"


def run(checkpoint: str, *, stages: int = 4, tokens: int = 24, prompt: list[int] | None = None,
        workdir: str | None = None, seed: int = 2) -> dict:
    from ..model_io.loader import checkpoint_config
    checkpoint = str(Path(checkpoint).expanduser().resolve())   # the commands run from the repo root
    cfg = checkpoint_config(checkpoint)
    if prompt is None:
        prompt = torch.randint(0, cfg.vocab_size, (12,),
                               generator=torch.Generator().manual_seed(seed)).tolist()
    tmp = Path(workdir or tempfile.mkdtemp(prefix="swarm-real-loopback-"))
    coord = tmp / "coord"
    port = _free_pair()
    agents = []
    t0 = time.perf_counter()
    _swarm("cluster", "create", "real-loopback", "--host", "127.0.0.1", "--port", str(port),
           "--state-dir", str(coord), "--json")
    try:
        _swarm("cluster", "start", "--state-dir", str(coord))
        for i in range(stages):
            st = tmp / f"node{i}"
            uri = _swarm("cluster", "pair", "--state-dir", str(coord)).strip().splitlines()[-1]
            _swarm("node", "join", uri, "--name", f"node{i}", "--state-dir", str(st))
            ready = tmp / f"node{i}.ready"
            agents.append((subprocess.Popen(
                [sys.executable, "-m", "swarm_inference_lab_b200.cli", "node", "agent",
                 "--state-dir", str(st), "--ready-file", str(ready)],
                env=_env(), cwd=ROOT, stdout=subprocess.DEVNULL, stderr=subprocess.PIPE,
                start_new_session=True), ready))
        for proc, ready in agents:
            t1 = time.time()
            while not ready.exists():
                if proc.poll() is not None:
                    raise RuntimeError(f"node agent exited: {proc.stderr.read().decode()[-2000:]}")
                if time.time() - t1 > 120:
                    raise RuntimeError("node agent did not become ready")
                time.sleep(0.1)
        out = _swarm("run", str(checkpoint), "--require-distributed", "--stages", str(stages),
                     "--prompt-ids", ",".join(map(str, prompt)), "--max-tokens", str(tokens),
                     "--json", "--state-dir", str(coord), timeout=600)
        res = json.loads(out.strip().splitlines()[-1])
    finally:
        for proc, _ in agents:
            if proc.poll() is None:
                try:
                    os.killpg(proc.pid, signal.SIGTERM)
                except ProcessLookupError:
                    pass
        for proc, _ in agents:
            try:
                proc.wait(timeout=20)
            except subprocess.TimeoutExpired:
                os.killpg(proc.pid, signal.SIGKILL)
                proc.wait(timeout=10)
        subprocess.run([sys.executable, "-m", "swarm_inference_lab_b200.cli", "cluster", "stop",
                        "--state-dir", str(coord)], env=_env(), cwd=ROOT, capture_output=True,
                       timeout=60)
    ref, ref_kind = reference_tokens(str(checkpoint), prompt, tokens)
    return {"checkpoint": str(checkpoint), "family": cfg.family, "stages": [
                {"layers": s["layers"], "worker": s["worker_id"]} for s in res["deployment"]["stages"]],
            "prompt": prompt, "tokens": res["tokens"], "reference_tokens": ref,
            "reference": ref_kind, "exact": res["tokens"] == ref,
            "stop_reason": res.get("stop_reason"), "distributed": res.get("distributed"),
            "seconds": time.perf_counter() - t0}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("checkpoint")
    ap.add_argument("--stages", type=int, default=4)
    ap.add_argument("--tokens", type=int, default=24)
    ap.add_argument("--out", default=None)
    a = ap.parse_args(argv)
    rep = run(a.checkpoint, stages=a.stages, tokens=a.tokens)
    if a.out:
        Path(a.out).write_text(json.dumps(rep, indent=1))
    print(json.dumps(rep))
    return 0 if rep["exact"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
