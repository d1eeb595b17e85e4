"""Duplicate-audit integrity checks, worker reputation and quarantine.

A sampled fraction of stage executions is re-run on a second worker; the two
outputs are compared exactly (token ids, hashes) or within a tolerance (hidden
states).  Agreement raises a worker's reputation slowly, disagreement lowers both
workers' reputations and, past a threshold or on repeated strikes, quarantines the
worker whose result disagrees with a third opinion (or with the higher-reputation
peer when there is none).  Quarantined workers are excluded from placement.

Reference: si/coordinator/integrity.py:22-78 (duplicate audits) and
si/security/reputation.py:16-67 (reputation / quarantine).
"""
from __future__ import annotations

import hashlib
import random
import time
from dataclasses import dataclass, field

import torch


@dataclass
class Reputation:
    score: float = 1.0
    audits: int = 0
    mismatches: int = 0
    quarantined: bool = False
    quarantined_at: float = 0.0
    history: list = field(default_factory=list)


class ReputationBook:
    def __init__(self, *, reward: float = 0.01, penalty: float = 0.25, floor: float = 0.5,
                 max_mismatches: int = 3):
        self.reward, self.penalty, self.floor, self.max_mismatches = reward, penalty, floor, max_mismatches
        self.workers: dict[str, Reputation] = {}

    def get(self, wid: str) -> Reputation:
        return self.workers.setdefault(wid, Reputation())

    def agree(self, wid: str) -> None:
        r = self.get(wid)
        r.audits += 1
        r.score = min(1.0, r.score + self.reward)

    def disagree(self, wid: str, reason: str) -> None:
        r = self.get(wid)
        r.audits += 1
        r.mismatches += 1
        r.score = max(0.0, r.score - self.penalty)
        r.history.append((time.time(), reason))
        if r.score < self.floor or r.mismatches >= self.max_mismatches:
            r.quarantined = True
            r.quarantined_at = time.time()

    def eligible(self, wid: str) -> bool:
        return not self.get(wid).quarantined

    def release(self, wid: str) -> None:
        r = self.get(wid)
        r.quarantined = False
        r.mismatches = 0
        r.score = self.floor


def digest(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().contiguous().cpu().numpy().tobytes()).hexdigest()


def outputs_match(a, b, *, exact: bool, rtol: float = 1e-2, atol: float = 1e-3) -> bool:
    if isinstance(a, torch.Tensor) and isinstance(b, torch.Tensor):
        if a.shape != b.shape or a.dtype != b.dtype:
            return False
        if exact:
            return digest(a) == digest(b)
        return bool(torch.allclose(a.float(), b.float(), rtol=rtol, atol=atol))
    return a == b


class IntegrityCoordinator:
    """Decides which executions to audit and applies the verdicts to reputations."""

    def __init__(self, book: ReputationBook | None = None, *, sample_rate: float = 0.05, seed: int = 0):
        self.book = book or ReputationBook()
        self.rate = sample_rate
        self.rng = random.Random(seed)
        self.log: list[dict] = []

    def should_audit(self) -> bool:
        return self.rng.random() < self.rate

    def judge(self, primary: str, primary_out, auditor: str, audit_out, *, exact: bool = True,
              tiebreak: tuple[str, object] | None = None) -> bool:
        ok = outputs_match(primary_out, audit_out, exact=exact)
        entry = {"primary": primary, "auditor": auditor, "match": ok, "t": time.time()}
        if ok:
            self.book.agree(primary)
            self.book.agree(auditor)
        else:
            if tiebreak is not None:
                third, third_out = tiebreak
                bad = primary if outputs_match(third_out, audit_out, exact=exact) else auditor
                entry["third"] = third
            else:
                bad = primary if self.book.get(primary).score <= self.book.get(auditor).score else auditor
            self.book.disagree(bad, f"mismatch vs {auditor if bad == primary else primary}")
            entry["blamed"] = bad
        self.log.append(entry)
        return ok
