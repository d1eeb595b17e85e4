"""Acceptance gates: the pre-physical software gate and the model matrix.

``pre_physical_gate`` runs the checks that need no GPU and must pass before any
hardware run: stage-ring golden vectors (Python and C++ codecs agree), the CPU
loopback pipeline matches a single-process run, the planner produces an admissible
plan for every benchmark preset, and every preset's parameter count and per-GPU
memory fit are consistent.  ``model_matrix`` reports, per preset, whether a plan fits
on one 8 x B200 box, its parallel layout and predicted throughput.  Both return JSON
evidence records (``write_evidence`` stores them with a timestamp and git revision).

Reference: si/acceptance/pre_physical.py, si/acceptance/productization.py,
si/acceptance/major_models.py.
"""
from __future__ import annotations

import json
import subprocess
import time
from pathlib import Path


def _check(name, fn) -> dict:
    t0 = time.perf_counter()
    try:
        detail = fn()
        return {"check": name, "ok": True, "detail": detail, "s": round(time.perf_counter() - t0, 3)}
    except Exception as exc:  # noqa: BLE001 - the verdict is the record
        return {"check": name, "ok": False, "detail": f"{type(exc).__name__}: {exc}",
                "s": round(time.perf_counter() - t0, 3)}


def _codec_agreement():
    from ..protocol import stage_ring as sr
    msg = sr.StageMessage(operation=sr.Operation.DECODE, model_revision="m", tokenizer_revision="t",
                          topology_id="topo", stage_id=0, layer_start=0, layer_end=2, session_id="s",
                          request_id="r", sequence_number=1, token_position=3, source_stage=0,
                          destination_stage=1, payload=b"\x01\x02")
    py = sr.encode(msg)
    assert sr.decode(py).payload == b"\x01\x02"
    try:
        from .. import _native
    except ImportError:
        return "python codec (native library not built)"
    op, flags, seq, pos, src, dst, meta, payload = _native.ring_decode(py)
    assert (seq, pos, payload) == (1, 3, b"\x01\x02")
    return "python and native codecs agree"


def _plans_for_presets():
    from ..engines import ClusterCapabilities, RequestShape
    from ..models.config import PRESETS
    from ..runtime.canonical import CanonicalRuntime
    rt = CanonicalRuntime()
    caps = ClusterCapabilities(nodes={"local": {"gpus": 8, "gpu_name": "NVIDIA B200"}})
    out = {}
    for name in PRESETS:
        r = rt.dry_run(name, caps, RequestShape(batch=32, prompt_tokens=1024, output_tokens=128,
                                                mode="throughput"))
        out[name] = r["winner"]["plan"] if r["winner"] else f"no plan: {r['rejected']}"
    return out


def pre_physical_gate() -> dict:
    checks = [_check("stage_ring_codec", _codec_agreement), _check("plans_for_presets", _plans_for_presets)]
    return {"gate": "pre_physical", "ok": all(c["ok"] for c in checks), "checks": checks}


def model_matrix(gpus: int = 8) -> list[dict]:
    from ..models.config import PRESETS
    from ..planner.box_planner import BoxMeasurements, plan_box
    rows = []
    m = BoxMeasurements()
    for name, cfg in PRESETS.items():
        plans = plan_box(cfg, gpus, m, batch=32, ctx=2048, prompt=1024, mode="throughput")
        fit = [p for p in plans if p.fits]
        best = fit[0] if fit else None
        rows.append({"model": name, "params": cfg.parameter_count(), "fits": bool(best),
                     "layout": None if best is None else f"tp{best.tp} ep{best.ep} pp{best.pp} dp{best.dp}",
                     "predicted_tok_s": None if best is None else round(best.tokens_per_s, 1)})
    return rows


def write_evidence(record: dict, out_dir: str | Path) -> Path:
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    try:
        rev = subprocess.run(["git", "rev-parse", "HEAD"], capture_output=True, text=True,
                             timeout=10).stdout.strip()
    except (OSError, subprocess.SubprocessError):
        rev = "unknown"
    record = dict(record, recorded_at=time.time(), git_revision=rev)
    p = out / f"{record.get('gate', 'evidence')}-{int(record['recorded_at'])}.json"
    p.write_text(json.dumps(record, indent=1, default=str))
    return p
