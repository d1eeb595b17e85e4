"""Exact stage-input replay log and request store.

Every token a session accepted is appended (with its position) to a per-request
log, so a stage that lost its KV cache can be rebuilt by replaying the prompt plus
the accepted tokens through a fresh owner (restart-and-replay).  The log is an
append-only JSON-lines file per request plus an in-memory index; entries carry a
running SHA-256 so a truncated or edited log is detected before it is replayed.

Reference: si/coordinator/replay_log.py:26 and si/coordinator/request_state.py:11.
"""
from __future__ import annotations

import hashlib
import json
from dataclasses import dataclass, field
from pathlib import Path


class ReplayLogError(RuntimeError):
    pass


@dataclass
class RequestRecord:
    request_id: str
    prompt: list[int]
    tokens: list[int] = field(default_factory=list)
    state: str = "running"
    chain: str = ""


def _link(prev: str, kind: str, value) -> str:
    return hashlib.sha256(f"{prev}|{kind}|{json.dumps(value)}".encode()).hexdigest()


class ReplayLog:
    def __init__(self, root: str | Path):
        self.root = Path(root)
        self.root.mkdir(parents=True, exist_ok=True)
        self.records: dict[str, RequestRecord] = {}

    def _path(self, rid: str) -> Path:
        return self.root / f"{rid}.jsonl"

    def _append(self, rid: str, entry: dict) -> None:
        with open(self._path(rid), "a") as f:
            f.write(json.dumps(entry) + "\n")
            f.flush()

    def open(self, rid: str, prompt: list[int]) -> RequestRecord:
        if rid in self.records or self._path(rid).exists():
            raise ReplayLogError(f"request {rid} already logged")
        rec = RequestRecord(rid, list(prompt))
        rec.chain = _link("", "prompt", rec.prompt)
        self._append(rid, {"kind": "prompt", "value": rec.prompt, "chain": rec.chain})
        self.records[rid] = rec
        return rec

    def accept(self, rid: str, position: int, token: int) -> None:
        rec = self.records[rid]
        expect = len(rec.prompt) + len(rec.tokens)
        if position != expect:
            raise ReplayLogError(f"request {rid}: token at position {position}, expected {expect}")
        rec.tokens.append(int(token))
        rec.chain = _link(rec.chain, "token", [position, int(token)])
        self._append(rid, {"kind": "token", "value": [position, int(token)], "chain": rec.chain})

    def finish(self, rid: str, state: str = "finished") -> None:
        rec = self.records[rid]
        rec.state = state
        rec.chain = _link(rec.chain, "state", state)
        self._append(rid, {"kind": "state", "value": state, "chain": rec.chain})

    def replay_inputs(self, rid: str) -> list[int]:
        """Token ids a fresh stage must consume to rebuild the request's KV state."""
        rec = self.records[rid]
        return rec.prompt + rec.tokens

    def load(self, rid: str) -> RequestRecord:
        """Rebuild a record from disk, verifying the hash chain."""
        rec = None
        chain = ""
        with open(self._path(rid)) as f:
            for line in f:
                e = json.loads(line)
                chain = _link(chain, e["kind"], e["value"])
                if chain != e["chain"]:
                    raise ReplayLogError(f"request {rid}: replay log chain broken")
                if e["kind"] == "prompt":
                    rec = RequestRecord(rid, list(e["value"]))
                elif e["kind"] == "token":
                    rec.tokens.append(int(e["value"][1]))
                else:
                    rec.state = e["value"]
        if rec is None:
            raise ReplayLogError(f"request {rid}: empty replay log")
        rec.chain = chain
        self.records[rid] = rec
        return rec
