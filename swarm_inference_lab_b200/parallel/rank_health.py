"""Host-side failure detection for the ranks of one job (one process per GPU).

Every rank runs a ``RankMonitor``: a daemon thread bumps the rank's heartbeat counter in the
job's key-value store (``torch.distributed`` ``TCPStore``, its own client connection) every
``interval_s``.  Between steps -- never with a kernel or collective in flight -- a rank calls
``check()``; it raises ``RankFailure`` naming the ranks that

* announced a failure (``fail(reason)``, from an exception handler, with the reason),
* left (``leave()``, an orderly exit between steps), or
* went silent (no heartbeat advance for ``timeout_s``: a crash or a kill).

A collective that a dead peer never joins ends with an error through the process group's own
short timeout (or the transport's reset); ``guard()`` wraps such a call and turns the error
into a ``RankFailure`` that names the silent ranks.  ``RankMonitor.start`` waits (bounded) for
every rank's first heartbeat, so a rank that never joins is reported too.

The monitor is the host half of the failure story; on the device every wait is bounded and
reports a status word (``csrc/include/sil/ptx.cuh``).

Reference: si/worker/runtime.py heartbeats and si/coordinator/service.py:662 (``heartbeat``:
a silent worker is marked failed) -- the same rule applied to the ranks of one box.
"""
from __future__ import annotations

import contextlib
import threading
import time
from datetime import timedelta


class RankFailure(RuntimeError):
    def __init__(self, ranks: dict[int, str]):
        self.ranks = dict(sorted(ranks.items()))
        super().__init__("rank failure: " + ", ".join(f"{r} ({why})" for r, why in self.ranks.items()))


class RankMonitor:
    def __init__(self, host: str, port: int, rank: int, world: int, *, prefix: str = "health",
                 interval_s: float = 0.2, timeout_s: float = 2.0):
        import torch.distributed as dist
        self.rank, self.world, self.prefix = rank, world, prefix
        self.interval_s, self.timeout_s = interval_s, timeout_s
        # two client connections: the heartbeat thread never shares one with the checks
        self._hb_store = dist.TCPStore(host, port, world_size=None, is_master=False,
                                       timeout=timedelta(seconds=30))
        self._store = dist.TCPStore(host, port, world_size=None, is_master=False,
                                    timeout=timedelta(seconds=30))
        self._seen: dict[int, tuple[int, float]] = {}   # rank -> (counter, when it last moved)
        self._stop = threading.Event()
        self._thread: threading.Thread | None = None

    def _key(self, kind: str, rank: int) -> str:
        return f"{self.prefix}/{kind}/{rank}"

    def _counter(self, rank: int) -> int:
        return int(self._store.add(self._key("hb", rank), 0))

    def _beat(self) -> None:
        while not self._stop.is_set():
            try:
                self._hb_store.add(self._key("hb", self.rank), 1)
            except Exception:  # noqa: BLE001 - the store is gone: the job is ending
                return
            self._stop.wait(self.interval_s)

    def start(self, join_timeout_s: float = 10.0) -> "RankMonitor":
        """Starts heartbeating and waits until every rank has beaten once; raises
        ``RankFailure`` for ranks that did not join in time."""
        self._thread = threading.Thread(target=self._beat, daemon=True, name=f"rank{self.rank}-hb")
        self._thread.start()
        t0 = time.monotonic()
        while True:
            missing = [r for r in range(self.world) if self._counter(r) == 0]
            if not missing:
                break
            if time.monotonic() - t0 > join_timeout_s:
                raise RankFailure({r: "never joined" for r in missing})
            time.sleep(self.interval_s / 2)
        now = time.monotonic()
        self._seen = {r: (self._counter(r), now) for r in range(self.world)}
        return self

    def fail(self, reason: str) -> None:
        """Announces this rank's failure (call from an exception handler, then exit)."""
        with contextlib.suppress(Exception):
            self._store.set(self._key("failed", self.rank), reason[:500])

    def leave(self) -> None:
        """An orderly exit between steps: the others stop at their next ``check``."""
        with contextlib.suppress(Exception):
            self._store.set(self._key("left", self.rank), "left")
        self.stop()

    def _flag(self, kind: str, rank: int) -> str | None:
        key = self._key(kind, rank)
        if self._store.check([key]):
            return self._store.get(key).decode(errors="replace")
        return None

    def failures(self) -> dict[int, str]:
        """Peers that failed, left or went silent, with the reason."""
        out = {}
        now = time.monotonic()
        for r in range(self.world):
            if r == self.rank:
                continue
            why = self._flag("failed", r)
            if why is not None:
                out[r] = f"failed: {why}"
                continue
            if self._flag("left", r) is not None:
                out[r] = "left"
                continue
            c = self._counter(r)
            last_c, last_t = self._seen.get(r, (c, now))
            if c != last_c:
                self._seen[r] = (c, now)
            elif now - last_t > self.timeout_s:
                out[r] = f"silent for {now - last_t:.1f} s"
        return out

    def check(self) -> None:
        """Raises ``RankFailure`` if a peer failed, left or went silent (call between steps)."""
        bad = self.failures()
        if bad:
            raise RankFailure(bad)

    @contextlib.contextmanager
    def guard(self, settle_s: float | None = None):
        """Runs a collective; if it raises, waits until a silent peer is recognisable (at most
        ``timeout_s`` + ``settle_s``) and raises ``RankFailure`` naming the failed ranks."""
        try:
            yield
        except RankFailure:
            raise
        except Exception as exc:  # noqa: BLE001 - a collective broken by a peer
            t0 = time.monotonic()
            limit = self.timeout_s + (settle_s if settle_s is not None else 2 * self.interval_s)
            while time.monotonic() - t0 <= limit + self.interval_s:
                bad = self.failures()
                if bad:
                    raise RankFailure(bad) from exc
                time.sleep(self.interval_s)
            raise

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2 * self.interval_s + 1.0)
