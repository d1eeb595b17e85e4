"""Process metrics and structured logs.

* ``Metrics``: named counters, gauges and latency summaries (count, sum, p50 / p99 over a
  bounded window), with optional labels, exported as a JSON snapshot and in the Prometheus
  text exposition format.  The coordinator counts registrations, heartbeats, lost workers,
  requests, tokens, recoveries and transport errors; stage owners count frames, rejected
  frames, backpressure refusals, relayed frames and forward time; the worker runtime counts
  heartbeats and control calls.  ``METRICS`` is the process-wide instance.
* ``JsonLogFormatter``: one JSON object per log line (time, level, logger, message and
  any ``extra=`` fields), for log shippers; ``configure_json_logging`` installs it.

Reference: si/runtime/telemetry.py (request and connection metrics, JSON event logs).
"""
from __future__ import annotations

import json
import logging
import threading
import time
from collections import deque


def _key(name: str, labels: dict | None) -> tuple:
    return (name, tuple(sorted((labels or {}).items())))


class Metrics:
    def __init__(self, window: int = 2048):
        self._lock = threading.Lock()
        self.counters: dict[tuple, float] = {}
        self.gauges: dict[tuple, float] = {}
        self.samples: dict[tuple, deque] = {}
        self.sums: dict[tuple, tuple[int, float]] = {}
        self.window = window
        self.started = time.time()

    def inc(self, name: str, value: float = 1.0, **labels) -> None:
        k = _key(name, labels)
        with self._lock:
            self.counters[k] = self.counters.get(k, 0.0) + value

    def set(self, name: str, value: float, **labels) -> None:
        with self._lock:
            self.gauges[_key(name, labels)] = float(value)

    def observe(self, name: str, value: float, **labels) -> None:
        k = _key(name, labels)
        with self._lock:
            d = self.samples.setdefault(k, deque(maxlen=self.window))
            d.append(float(value))
            n, s = self.sums.get(k, (0, 0.0))
            self.sums[k] = (n + 1, s + float(value))

    def counter(self, name: str, **labels) -> float:
        return self.counters.get(_key(name, labels), 0.0)

    @staticmethod
    def _quantile(xs: list[float], q: float) -> float:
        if not xs:
            return 0.0
        ys = sorted(xs)
        return ys[min(len(ys) - 1, int(q * (len(ys) - 1) + 0.5))]

    def snapshot(self) -> dict:
        with self._lock:
            out = {"uptime_s": time.time() - self.started, "counters": {}, "gauges": {},
                   "summaries": {}}
            for (n, lb), v in self.counters.items():
                out["counters"][n + _fmt_labels(lb)] = v
            for (n, lb), v in self.gauges.items():
                out["gauges"][n + _fmt_labels(lb)] = v
            for k, d in self.samples.items():
                n, lb = k
                cnt, s = self.sums[k]
                xs = list(d)
                out["summaries"][n + _fmt_labels(lb)] = {
                    "count": cnt, "sum": s, "p50": self._quantile(xs, 0.5),
                    "p99": self._quantile(xs, 0.99)}
            return out

    def prometheus(self, prefix: str = "swarm_") -> str:
        """Prometheus text exposition (counters, gauges, summaries with p50 / p99)."""
        lines = []
        with self._lock:
            for (n, lb), v in sorted(self.counters.items()):
                lines.append(f"{prefix}{n}_total{_fmt_labels(lb)} {v:g}")
            for (n, lb), v in sorted(self.gauges.items()):
                lines.append(f"{prefix}{n}{_fmt_labels(lb)} {v:g}")
            for k in sorted(self.samples):
                n, lb = k
                cnt, s = self.sums[k]
                xs = list(self.samples[k])
                for q in (0.5, 0.99):
                    lines.append(f"{prefix}{n}{_fmt_labels(lb + (('quantile', str(q)),))} "
                                 f"{self._quantile(xs, q):g}")
                lines.append(f"{prefix}{n}_count{_fmt_labels(lb)} {cnt}")
                lines.append(f"{prefix}{n}_sum{_fmt_labels(lb)} {s:g}")
        return "\n".join(lines) + "\n"


def _fmt_labels(lb: tuple) -> str:
    if not lb:
        return ""
    return "{" + ",".join(f'{k}="{v}"' for k, v in lb) + "}"


METRICS = Metrics()


class JsonLogFormatter(logging.Formatter):
    _skip = set(vars(logging.makeLogRecord({})).keys()) | {"message", "asctime"}

    def format(self, record: logging.LogRecord) -> str:
        out = {"ts": round(record.created, 6), "level": record.levelname, "logger": record.name,
               "msg": record.getMessage()}
        for k, v in vars(record).items():
            if k not in self._skip and not k.startswith("_"):
                try:
                    json.dumps(v)
                    out[k] = v
                except (TypeError, ValueError):
                    out[k] = repr(v)
        if record.exc_info:
            out["exc"] = self.formatException(record.exc_info)
        return json.dumps(out, sort_keys=True)


def configure_json_logging(level: int = logging.INFO, stream=None) -> logging.Handler:
    h = logging.StreamHandler(stream)
    h.setFormatter(JsonLogFormatter())
    root = logging.getLogger("swarm")
    root.addHandler(h)
    root.setLevel(level)
    return h
