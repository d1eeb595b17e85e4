"""Device timing and clock sampling used by the benchmarks.

Timing rule: CUDA events on the launching stream, after warm-up, with a
synchronize on both sides; multi-GPU numbers take the max over ranks.
``ClockSampler`` polls ``nvidia-smi`` (read-only queries) during a timed
region and summarises SM clocks and active throttle reasons.
"""
from __future__ import annotations

import csv
import io
import shutil
import statistics
import subprocess
import threading

import torch


class EventTimer:
    def __init__(self):
        self.start = torch.cuda.Event(enable_timing=True)
        self.end = torch.cuda.Event(enable_timing=True)

    def __enter__(self):
        torch.cuda.synchronize()
        self.start.record()
        return self

    def __exit__(self, *exc):
        self.end.record()
        torch.cuda.synchronize()

    @property
    def ms(self) -> float:
        return self.start.elapsed_time(self.end)


QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


class ClockSampler:
    """Samples SM clock and throttle reasons of one GPU every ``period_ms`` (read-only)."""

    def __init__(self, gpu_index: int, period_ms: int = 200):
        self.gpu = gpu_index
        self.period = period_ms / 1000.0
        self.rows: list[dict] = []
        self._stop = threading.Event()
        self._thr: threading.Thread | None = None
        self.available = shutil.which("nvidia-smi") is not None

    def _poll(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={QUERY}",
                                      "--format=csv,noheader,nounits"], capture_output=True,
                                     text=True, timeout=5).stdout
                for row in csv.reader(io.StringIO(out)):
                    if len(row) >= 9:
                        self.rows.append([c.strip() for c in row])
            except Exception:
                pass
            self._stop.wait(self.period)

    def __enter__(self):
        if self.available:
            self._thr = threading.Thread(target=self._poll, daemon=True)
            self._thr.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thr is not None:
            self._thr.join(timeout=10)

    def summary(self) -> dict:
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        sm = [num(r[1]) for r in self.rows if num(r[1]) is not None]
        mx = [num(r[2]) for r in self.rows if num(r[2]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4)
                          if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.rows)}
