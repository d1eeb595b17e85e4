"""Engine capabilities and the probe-generated compatibility registry.

``engine_facts`` turns a worker's capability report (``worker_caps.local_capabilities``)
into the facts engines are matched on: compute capability, whether the sm_100a
kernels can run, dtypes the tensor cores take (bf16, fp8 e4m3), device memory and
peer access.  ``CompatibilityRegistry`` records, per (engine, model family, weight
dtype, device class), whether a probe run passed and why not; the planner consults
it before proposing an engine for a model (a failed probe rejects the pair with its
reason; an unprobed pair is allowed with reduced confidence).

Reference: si/engines/capabilities.py:68,102; si/engines/compatibility.py:138;
si/engines/local_capabilities.py:378.
"""
from __future__ import annotations

import json
import time
from dataclasses import asdict, dataclass
from pathlib import Path


def engine_facts(caps: dict) -> dict:
    devs = caps.get("devices", [])
    ccs = [tuple(int(x) for x in d.get("capability", "0.0").split(".")) for d in devs]
    sm100 = bool(ccs) and all(c[0] == 10 for c in ccs)
    return {
        "gpus": len(devs),
        "device_class": "b200" if sm100 else ("gpu" if devs else "cpu"),
        "sm100a_kernels": sm100,
        "dtypes": (["bf16", "fp8_e4m3", "fp32"] if sm100 else ["fp32"]),
        "device_memory_gb": [d.get("memory_gb", 0) for d in devs],
        "min_device_memory_gb": min((d.get("memory_gb", 0) for d in devs), default=0),
        "host_memory_gb": caps.get("host_memory_gb", 0),
        "cpus": caps.get("cpus", 0),
    }


@dataclass
class CompatRecord:
    engine: str
    family: str
    weight_dtype: str
    device_class: str
    ok: bool
    reason: str = ""
    probed_at: float = 0.0
    evidence: str = ""        # e.g. the test or bench that produced the verdict


class CompatibilityRegistry:
    def __init__(self, path: str | Path | None = None):
        self.path = Path(path) if path else None
        self.records: dict[tuple, CompatRecord] = {}
        if self.path and self.path.exists():
            for r in json.loads(self.path.read_text()):
                rec = CompatRecord(**r)
                self.records[self._k(rec.engine, rec.family, rec.weight_dtype, rec.device_class)] = rec

    @staticmethod
    def _k(engine, family, dtype, dev):
        return (engine, family, dtype, dev)

    def record(self, engine: str, family: str, weight_dtype: str, device_class: str, ok: bool,
               reason: str = "", evidence: str = "") -> CompatRecord:
        rec = CompatRecord(engine, family, weight_dtype, device_class, ok, reason, time.time(), evidence)
        self.records[self._k(engine, family, weight_dtype, device_class)] = rec
        if self.path:
            self.path.write_text(json.dumps([asdict(r) for r in self.records.values()], indent=1))
        return rec

    def check(self, engine: str, family: str, weight_dtype: str, device_class: str) -> tuple[bool, str, float]:
        """(allowed, reason, confidence factor)."""
        rec = self.records.get(self._k(engine, family, weight_dtype, device_class))
        if rec is None:
            return True, "unprobed", 0.9
        return rec.ok, rec.reason or "probed", 1.0 if rec.ok else 0.0


def probe_native_stage(registry: CompatibilityRegistry, facts: dict, family: str, weight_dtype: str,
                       run_probe) -> CompatRecord:
    """Run ``run_probe()`` (a tiny forward on the device, raising on failure) and record it."""
    if not facts["sm100a_kernels"]:
        return registry.record("native-stage", family, weight_dtype, facts["device_class"], False,
                               "sm_100a kernels need compute capability 10.x")
    if weight_dtype.startswith("fp8") and "fp8_e4m3" not in facts["dtypes"]:
        return registry.record("native-stage", family, weight_dtype, facts["device_class"], False,
                               "no e4m3 tensor-core support")
    try:
        run_probe()
        return registry.record("native-stage", family, weight_dtype, facts["device_class"], True,
                               evidence="probe forward")
    except Exception as exc:  # noqa: BLE001 - the verdict is the product here
        return registry.record("native-stage", family, weight_dtype, facts["device_class"], False,
                               f"{type(exc).__name__}: {exc}"[:300])
