"""Coordinator-side model catalog built from worker probes.

The coordinator never loads weights: workers inspect model sources they can reach
(headers / configs only) and report ``{source, revision, family, bytes, layers,
runnable}``; the catalog keeps the latest report per (worker, source), answers which
workers hold a given revision, and resolves a request for a model name to the
revision most workers agree on (ties: newest report).

Reference: si/coordinator/model_catalog.py:66.
"""
from __future__ import annotations

import time
from collections import Counter
from dataclasses import dataclass, field


@dataclass
class ModelReport:
    worker_id: str
    source: str
    revision: str
    family: str
    bytes: int
    layers: int
    runnable: bool
    reported_at: float = field(default_factory=time.time)


class ModelCatalog:
    def __init__(self):
        self.reports: dict[tuple[str, str], ModelReport] = {}

    def report(self, r: ModelReport) -> None:
        self.reports[(r.worker_id, r.source)] = r

    def forget_worker(self, worker_id: str) -> None:
        for k in [k for k in self.reports if k[0] == worker_id]:
            del self.reports[k]

    def holders(self, revision: str) -> list[str]:
        return sorted({r.worker_id for r in self.reports.values() if r.revision == revision})

    def resolve(self, source: str) -> ModelReport | None:
        cands = [r for r in self.reports.values() if r.source == source and r.runnable]
        if not cands:
            return None
        votes = Counter(r.revision for r in cands)
        best = max(votes.values())
        top = [r for r in cands if votes[r.revision] == best]
        return max(top, key=lambda r: r.reported_at)

    def listing(self) -> list[dict]:
        out: dict[str, dict] = {}
        for r in self.reports.values():
            e = out.setdefault(r.revision, {"source": r.source, "revision": r.revision,
                                            "family": r.family, "bytes": r.bytes, "layers": r.layers,
                                            "workers": []})
            e["workers"].append(r.worker_id)
        for e in out.values():
            e["workers"].sort()
        return sorted(out.values(), key=lambda e: e["source"])


def probe_report(worker_id: str, source: str) -> ModelReport:
    """What a worker reports for ``source`` (inspection only, no weights)."""
    from ..runtime.canonical import CanonicalRuntime
    try:
        info = CanonicalRuntime().inspect(source)
        return ModelReport(worker_id, source, info["revision"], info["family"], int(info.get("bytes", 0)),
                           int(info["layers"]), True)
    except Exception:  # noqa: BLE001 - unreadable sources are reported as not runnable
        return ModelReport(worker_id, source, "unknown", "unknown", 0, 0, False)
