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


# ---------------------------------------------------------------- frozen contracts
CONTRACTS = Path(__file__).resolve().parent / "contracts"


def _field(d: dict, path: str):
    cur = d
    for part in path.split("."):
        if not isinstance(cur, dict) or part not in cur:
            raise KeyError(path)
        cur = cur[part]
    return cur


def load_contract(name_or_path: str) -> dict:
    import yaml
    p = Path(name_or_path)
    if not p.exists():
        p = CONTRACTS / f"{name_or_path}.yaml"
    return yaml.safe_load(p.read_text())


def check_contract(contract: dict, evidence: dict) -> dict:
    """Evaluates every required field and gate of a frozen contract against an evidence
    record; returns ``{"contract", "ok", "results": [...]}`` (missing fields fail)."""
    ops = {"==": lambda a, b: a == b, ">=": lambda a, b: a >= b, ">": lambda a, b: a > b,
           "<=": lambda a, b: a <= b, "<": lambda a, b: a < b,
           "excludes_any": lambda a, b: not (set(a or []) & set(b))}
    results = []
    for f, want in (contract.get("required") or {}).items():
        try:
            got = _field(evidence, f)
            results.append({"field": f, "ok": got == want, "got": got, "want": want})
        except KeyError:
            results.append({"field": f, "ok": False, "got": None, "want": want})
    for g in contract.get("gates") or []:
        try:
            got = _field(evidence, g["field"])
            ok = bool(ops[g["op"]](got, g["value"]))
        except (KeyError, TypeError):
            got, ok = None, False
        results.append({"field": g["field"], "op": g["op"], "ok": ok, "got": got, "want": g["value"]})
    return {"contract": contract.get("name"), "ok": all(r["ok"] for r in results),
            "results": results}


def main(argv=None):
    """``python -m swarm_inference_lab_b200.testing.acceptance CONTRACT EVIDENCE.json``: checks
    the last JSON object of the evidence file against the contract; exit 1 on failure."""
    import sys
    args = list(sys.argv[1:] if argv is None else argv)
    if len(args) != 2:
        print("usage: acceptance CONTRACT EVIDENCE.json", file=sys.stderr)
        return 2
    text = Path(args[1]).read_text().strip()
    ev = None
    for line in text.splitlines()[::-1]:
        if line.startswith("{"):
            ev = json.loads(line)
            break
    if ev is None:
        ev = json.loads(text)
    rep = check_contract(load_contract(args[0]), ev)
    print(json.dumps(rep, indent=1, default=str))
    return 0 if rep["ok"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
