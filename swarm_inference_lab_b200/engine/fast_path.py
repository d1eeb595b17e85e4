"""Exactness-gated fast-path ladder with measured selection and a persistent profile store.

Candidates are decode configurations of the same engine, from the most
conservative to the fastest:

    eager            kernels launched one by one, no programmatic dependent launch
    eager+pdl        ... with programmatic dependent launch
    graph+pdl        the whole decode step captured in a CUDA graph

Each candidate must reproduce the baseline's greedy tokens on a probe batch
(exactness gate); the passing candidates are timed on the device and the fastest
is selected.  The result is stored per (model, device, batch bucket) in a JSON
profile store so later processes reuse it without re-measuring.

Reference: si/model/qwen3_fast_path.py:29 (candidates and gates),
si/execution/fast_path_registry.py:25, si/runtime/performance_profiles.py:60.
"""
from __future__ import annotations

import json
import os
import time
from dataclasses import asdict, dataclass
from pathlib import Path

import torch


@dataclass(frozen=True)
class Candidate:
    name: str
    cuda_graphs: bool
    pdl: bool


LADDER = (Candidate("eager", False, False), Candidate("eager+pdl", False, True),
          Candidate("graph+pdl", True, True))


@dataclass
class FastPathResult:
    name: str
    exact: bool
    ms_per_step: float | None
    error: str = ""


class ProfileStore:
    def __init__(self, path: str | os.PathLike):
        self.path = Path(path)
        self.data = json.loads(self.path.read_text()) if self.path.exists() else {}

    @staticmethod
    def key(model: str, device: str, bucket: int) -> str:
        return f"{model}|{device}|b{bucket}"

    def get(self, key: str) -> dict | None:
        return self.data.get(key)

    def put(self, key: str, record: dict) -> None:
        self.data[key] = record
        tmp = self.path.with_suffix(".tmp")
        tmp.write_text(json.dumps(self.data, indent=1, sort_keys=True))
        os.replace(tmp, self.path)


def _set_pdl(on: bool) -> bool:
    from ..ops._ext import ext
    fn = getattr(ext(), "set_pdl", None)
    if fn is None:
        return False
    fn(bool(on))
    return True


def _run(make_engine, cand: Candidate, prompts, new_tokens: int, steps: int):
    pdl_ok = _set_pdl(cand.pdl)
    if cand.pdl and not pdl_ok:
        raise RuntimeError("this build cannot toggle programmatic dependent launch")
    eng = make_engine(cand.cuda_graphs)
    from .engine import SamplingParams
    outs, _ = eng.generate(prompts, SamplingParams(max_new_tokens=new_tokens))
    toks = [o.token_ids for o in outs]
    # device-timed decode steps on the chosen path
    from .runner import bucket_for
    dg = eng.runner.graph_for(bucket_for(len(prompts)))
    ids = [t[-1] for t in toks]
    pos = [len(p) + len(t) - 1 for p, t in zip(prompts, toks)]
    for p in prompts:
        eng.kv.open(f"fp{id(p)}")
    pages = []
    for p in prompts:
        s = eng.kv.reserve(f"fp{id(p)}", len(p) + new_tokens + steps + 2)
        pages.append(s.pages)
    eng.runner.stage_decode_inputs(dg, ids, pos, pages)
    for _ in range(2):
        eng.runner.replay(dg)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        eng.runner.replay(dg)
    b.record()
    torch.cuda.synchronize()
    for p in prompts:
        eng.kv.close(f"fp{id(p)}")
    return toks, a.elapsed_time(b) / steps


def select_fast_path(make_engine, prompts: list[list[int]], *, new_tokens: int = 8, steps: int = 16,
                     ladder=LADDER, store: ProfileStore | None = None, key: str | None = None) -> dict:
    """``make_engine(cuda_graphs: bool) -> LLMEngine``.  Returns the selection record."""
    if store is not None and key is not None and (rec := store.get(key)) is not None:
        return rec
    results: list[FastPathResult] = []
    baseline = None
    for cand in ladder:
        try:
            toks, ms = _run(make_engine, cand, prompts, new_tokens, steps)
        except Exception as exc:  # noqa: BLE001 - a failing candidate is recorded and skipped
            results.append(FastPathResult(cand.name, False, None, f"{type(exc).__name__}: {exc}"))
            continue
        if baseline is None:
            baseline = toks
        results.append(FastPathResult(cand.name, toks == baseline, ms))
    _set_pdl(True)
    passing = [r for r in results if r.exact and r.ms_per_step is not None]
    best = min(passing, key=lambda r: r.ms_per_step) if passing else None
    rec = {"selected": best.name if best else None, "measured_at": time.time(),
           "candidates": [asdict(r) for r in results]}
    if store is not None and key is not None:
        store.put(key, rec)
    return rec
