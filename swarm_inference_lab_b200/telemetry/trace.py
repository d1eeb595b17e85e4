"""Tracing and telemetry: JSONL span traces, critical-path reconstruction,
lifecycle events, and NVTX ranges.

* ``TraceWriter``: thread-safe JSONL writer of spans (``with tw.span(name, **attrs)``)
  and instant events; every record carries a monotonic timestamp, process
  and thread ids and optional causal parents (``after=[span ids]``).
* ``merge_traces`` merges per-process files by timestamp; ``chrome_trace`` converts records
  to the Chrome trace-event format (chrome://tracing, Perfetto): one row per process and
  thread, causal ``after`` links as flow arrows.
* ``critical_path`` walks the dependency graph backwards from the latest
  span and reports the chain that bounds end-to-end latency, counting
  token-critical receives (spans named ``recv*`` on the path).
* ``LifecycleObserver`` appends product events (session_opened,
  recovery_started, route_generation_installed, ...) to the file named by
  ``SWARM_LIFECYCLE_FILE`` when set.
* ``nvtx_range`` wraps ``torch.cuda.nvtx`` when enabled (off by default).

Reference: si/runtime/telemetry.py:614-900 (TraceWriter, merge_traces,
reconstruct_critical_path, lifecycle observer), si/model/qwen3_runtime.py:278-288.
"""
from __future__ import annotations

import contextlib
import itertools
import json
import os
import threading
import time
from pathlib import Path

_ids = itertools.count(1)


class TraceWriter:
    def __init__(self, path: str | Path | None, process: str = ""):
        self.path = Path(path) if path else None
        self.process = process or f"pid{os.getpid()}"
        self._lock = threading.Lock()
        self._f = open(self.path, "a", buffering=1) if self.path else None
        self.records: list[dict] = []

    def _write(self, rec: dict) -> None:
        with self._lock:
            self.records.append(rec)
            if self._f:
                self._f.write(json.dumps(rec, sort_keys=True) + "\n")

    def event(self, name: str, **attrs) -> int:
        sid = next(_ids)
        self._write({"id": f"{self.process}:{sid}", "kind": "event", "name": name,
                     "ts_ns": time.monotonic_ns(), "process": self.process,
                     "thread": threading.get_ident(), "attrs": attrs})
        return sid

    @contextlib.contextmanager
    def span(self, name: str, after: list[str] | None = None, **attrs):
        sid = f"{self.process}:{next(_ids)}"
        t0 = time.monotonic_ns()
        rec = {"id": sid, "kind": "span", "name": name, "start_ns": t0, "process": self.process,
               "thread": threading.get_ident(), "after": list(after or []), "attrs": attrs}
        try:
            yield sid
        finally:
            rec["end_ns"] = time.monotonic_ns()
            rec["dur_ms"] = (rec["end_ns"] - t0) / 1e6
            self._write(rec)

    def close(self) -> None:
        if self._f:
            self._f.close()
            self._f = None


def read_trace(path) -> list[dict]:
    return [json.loads(l) for l in Path(path).read_text().splitlines() if l.strip()]


def merge_traces(paths) -> list[dict]:
    recs = []
    for p in paths:
        recs.extend(read_trace(p))
    return sorted(recs, key=lambda r: r.get("start_ns", r.get("ts_ns", 0)))


def critical_path(records: list[dict]) -> dict:
    spans = {r["id"]: r for r in records if r.get("kind") == "span"}
    if not spans:
        return {"path": [], "total_ms": 0.0, "token_critical_receives": 0}
    cur = max(spans.values(), key=lambda r: r["end_ns"])
    path = [cur]
    while True:
        preds = [spans[p] for p in cur.get("after", []) if p in spans]
        if not preds:
            # implicit predecessor: the latest span ending before this one starts
            preds = [s for s in spans.values() if s["end_ns"] <= cur["start_ns"]]
        if not preds:
            break
        cur = max(preds, key=lambda r: r["end_ns"])
        path.append(cur)
    path.reverse()
    total = (path[-1]["end_ns"] - path[0]["start_ns"]) / 1e6
    recv = sum(1 for s in path if s["name"].startswith("recv"))
    return {"path": [s["name"] for s in path], "total_ms": total, "token_critical_receives": recv}


def chrome_trace(records: list[dict]) -> dict:
    """Chrome trace-event JSON of span / event records: spans become complete events ("X",
    microseconds), events instant events ("i"), each process a ``pid`` with its name, and each
    ``after`` dependency a flow arrow ("s" / "f") from the predecessor's end to the span."""
    pids: dict[str, int] = {}
    out: list[dict] = []
    spans = {r["id"]: r for r in records if r.get("kind") == "span"}
    for r in records:
        proc = r.get("process", "")
        if proc not in pids:
            pids[proc] = len(pids) + 1
            out.append({"ph": "M", "name": "process_name", "pid": pids[proc],
                        "args": {"name": proc}})
        base = {"name": r["name"], "pid": pids[proc], "tid": r.get("thread", 0),
                "args": dict(r.get("attrs") or {}, id=r["id"])}
        if r.get("kind") == "span":
            out.append(dict(base, ph="X", ts=r["start_ns"] / 1e3,
                            dur=(r["end_ns"] - r["start_ns"]) / 1e3))
        else:
            out.append(dict(base, ph="i", s="t", ts=r["ts_ns"] / 1e3))
    flow = 0
    for r in spans.values():
        for dep in r.get("after", []):
            src = spans.get(dep)
            if src is None:
                continue
            flow += 1
            out.append({"ph": "s", "id": flow, "name": "after", "cat": "dep",
                        "pid": pids[src.get("process", "")], "tid": src.get("thread", 0),
                        "ts": src["end_ns"] / 1e3})
            out.append({"ph": "f", "bp": "e", "id": flow, "name": "after", "cat": "dep",
                        "pid": pids[r.get("process", "")], "tid": r.get("thread", 0),
                        "ts": r["start_ns"] / 1e3})
    return {"traceEvents": out, "displayTimeUnit": "ms"}


def write_chrome_trace(paths, out_path) -> Path:
    """Merges JSONL trace files and writes them as one Chrome trace JSON file."""
    out = Path(out_path)
    out.write_text(json.dumps(chrome_trace(merge_traces(paths))))
    return out


class LifecycleObserver:
    def __init__(self, path: str | None = None):
        self.path = path or os.environ.get("SWARM_LIFECYCLE_FILE")
        self._lock = threading.Lock()

    def emit(self, event: str, **fields) -> None:
        if not self.path:
            return
        rec = {"event": event, "ts": time.time(), **fields}
        with self._lock, open(self.path, "a") as f:
            f.write(json.dumps(rec, sort_keys=True) + "\n")


@contextlib.contextmanager
def nvtx_range(name: str, enabled: bool = False):
    if not enabled:
        yield
        return
    import torch
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()
