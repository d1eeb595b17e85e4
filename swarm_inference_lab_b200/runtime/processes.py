"""Engine process lifecycle: hash-verified launch and bounded, signal-aware shutdown.

``EngineProcess`` starts a worker / engine command only after the files it will
execute match the SHA-256 digests recorded when the plan was made (a replaced
binary or module refuses to start), waits for its JSON ``ready`` line with a
deadline, and stops it with SIGTERM, then SIGKILL after a grace period.
``shutdown_all`` stops a set of processes concurrently within one deadline and
reports what each needed.  ``install_signal_handlers`` turns SIGTERM / SIGINT into
one orderly shutdown of everything registered.

Reference: si/runtime/engine_processes.py:64 and si/runtime/shutdown.py:11,60.
"""
from __future__ import annotations

import hashlib
import json
import os
import select
import signal
import subprocess
import time
from dataclasses import dataclass, field
from pathlib import Path


class ProcessVerificationError(RuntimeError):
    pass


def file_digest(path: str | os.PathLike) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for b in iter(lambda: f.read(1 << 20), b""):
            h.update(b)
    return h.hexdigest()


@dataclass
class EngineProcess:
    argv: list[str]
    verify: dict[str, str] = field(default_factory=dict)   # path -> expected sha256
    env: dict[str, str] | None = None
    cwd: str | None = None
    proc: subprocess.Popen | None = None
    ready: dict | None = None

    def check(self) -> None:
        for path, want in self.verify.items():
            if not Path(path).exists():
                raise ProcessVerificationError(f"{path} is missing")
            got = file_digest(path)
            if got != want:
                raise ProcessVerificationError(f"{path}: sha256 {got[:12]} != expected {want[:12]}")

    def start(self, ready_timeout_s: float = 60.0) -> dict:
        self.check()
        env = dict(os.environ, **(self.env or {}))
        self.proc = subprocess.Popen(self.argv, stdout=subprocess.PIPE, stderr=subprocess.PIPE,
                                     env=env, cwd=self.cwd, start_new_session=True, text=True)
        deadline = time.monotonic() + ready_timeout_s
        while time.monotonic() < deadline:
            if self.proc.poll() is not None:
                err = self.proc.stderr.read()[-2000:] if self.proc.stderr else ""
                raise RuntimeError(f"process exited with {self.proc.returncode} before ready: {err}")
            r, _, _ = select.select([self.proc.stdout], [], [], 0.1)
            if r:
                line = self.proc.stdout.readline()
                if line.startswith("{"):
                    msg = json.loads(line)
                    if msg.get("ready"):
                        self.ready = msg
                        return msg
        self.stop(grace_s=1.0)
        raise TimeoutError("process did not report ready in time")

    def alive(self) -> bool:
        return self.proc is not None and self.proc.poll() is None

    def stop(self, grace_s: float = 5.0) -> str:
        """SIGTERM the process group, SIGKILL after ``grace_s``.  Returns how it ended."""
        if self.proc is None or self.proc.poll() is not None:
            return "exited"
        try:
            os.killpg(self.proc.pid, signal.SIGTERM)
        except ProcessLookupError:
            return "exited"
        try:
            self.proc.wait(grace_s)
            return "terminated"
        except subprocess.TimeoutExpired:
            try:
                os.killpg(self.proc.pid, signal.SIGKILL)
            except ProcessLookupError:
                return "terminated"
            self.proc.wait(5.0)
            return "killed"


def shutdown_all(procs: list[EngineProcess], deadline_s: float = 10.0) -> list[str]:
    """Stop every process within one overall deadline (TERM all first, then KILL)."""
    for p in procs:
        if p.alive():
            try:
                os.killpg(p.proc.pid, signal.SIGTERM)
            except ProcessLookupError:
                pass
    end = time.monotonic() + deadline_s
    out = []
    for p in procs:
        if p.proc is None:
            out.append("never-started")
            continue
        left = max(0.0, end - time.monotonic())
        try:
            p.proc.wait(left)
            out.append("terminated")
        except subprocess.TimeoutExpired:
            out.append(p.stop(grace_s=0.0))
    return out


_registered: list[EngineProcess] = []


def install_signal_handlers(procs: list[EngineProcess], deadline_s: float = 10.0) -> None:
    _registered[:] = procs

    def handler(signum, frame):  # noqa: ARG001
        shutdown_all(_registered, deadline_s)
        raise SystemExit(128 + signum)

    signal.signal(signal.SIGTERM, handler)
    signal.signal(signal.SIGINT, handler)
