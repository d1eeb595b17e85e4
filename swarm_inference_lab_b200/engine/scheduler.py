"""Iteration-level continuous batching over a paged KV pool.

Each iteration returns a decode set (running sequences that get one token)
and a prefill set (waiting or partially prefilled sequences that get a chunk
of their prompt, bounded by a token budget).  Policies:

* ``latency``    - decode every runnable sequence, admit prefill only when
                   nothing is decoding or a request starves;
* ``balanced``   - decode, and give prefill the leftover token budget;
* ``throughput`` - prefill first (fill the batch), then decode.

Differences from the reference scheduler (si/worker/continuous_scheduler.py:79-286),
which admits only homogeneous prompt lengths into a static cache: prompts of
any length share one batch (varlen prefill over paged KV), admission is
bounded by free KV pages instead of a token count, and chunked prefill may
split one prompt over several iterations.  The starvation limit, the three
policy names and the per-iteration metrics follow the reference.
"""
from __future__ import annotations

import time
from collections import Counter, deque
from dataclasses import asdict, dataclass, field
from enum import Enum
from typing import Any


class SchedulerPolicy(str, Enum):
    LATENCY = "latency"
    BALANCED = "balanced"
    THROUGHPUT = "throughput"


@dataclass
class SeqRequest:
    request_id: str
    prompt: list[int]
    max_new_tokens: int
    admitted_ns: int
    admitted_iteration: int = 0
    prompt_consumed: int = 0
    output: list[int] = field(default_factory=list)
    last_served_iteration: int = -1
    finished: bool = False
    stop_token_ids: tuple[int, ...] = ()
    first_token_ns: int = 0
    finish_ns: int = 0
    sampling: object | None = None   # SamplingParams of a non-greedy request (None: greedy)

    @property
    def prefill_complete(self) -> bool:
        return self.prompt_consumed >= len(self.prompt)

    @property
    def context_len(self) -> int:
        return self.prompt_consumed + len(self.output)

    @property
    def remaining_prompt(self) -> int:
        return len(self.prompt) - self.prompt_consumed


@dataclass(frozen=True)
class Iteration:
    index: int
    decode: tuple[str, ...]
    prefill: tuple[tuple[str, int], ...]  # (request id, chunk tokens)
    starved: tuple[str, ...]
    overhead_ms: float


@dataclass
class SchedulerMetrics:
    iterations: int = 0
    overhead_ms: float = 0.0
    batch_size_distribution: Counter = field(default_factory=Counter)
    prefill_chunk_distribution: Counter = field(default_factory=Counter)
    starvation_events: int = 0
    maximum_wait_ms: float = 0.0
    useful_tokens: int = 0

    def payload(self) -> dict[str, Any]:
        p = asdict(self)
        p["batch_size_distribution"] = {str(k): v for k, v in sorted(self.batch_size_distribution.items())}
        p["prefill_chunk_distribution"] = {str(k): v for k, v in sorted(self.prefill_chunk_distribution.items())}
        return p


class ContinuousScheduler:
    def __init__(self, *, max_batch: int, prefill_token_budget: int, kv_capacity_tokens: int,
                 policy: SchedulerPolicy | str = SchedulerPolicy.BALANCED,
                 starvation_limit: int = 32, page_size: int = 64):
        if max_batch <= 0 or prefill_token_budget <= 0 or kv_capacity_tokens <= 0:
            raise ValueError("scheduler limits must be positive")
        self.policy = SchedulerPolicy(policy)
        self.max_batch = max_batch
        self.budget = prefill_token_budget
        self.kv_capacity = kv_capacity_tokens
        self.starvation_limit = starvation_limit
        self.page = page_size
        self.waiting: deque[SeqRequest] = deque()
        self.running: dict[str, SeqRequest] = {}
        self.iteration = 0
        self.metrics = SchedulerMetrics()

    # ------------------------------------------------------------ admission
    def admit(self, req: SeqRequest) -> None:
        if not req.request_id:
            raise ValueError("request_id cannot be empty")
        if req.request_id in self.running or any(r.request_id == req.request_id for r in self.waiting):
            raise ValueError(f"duplicate request {req.request_id!r}")
        if len(req.prompt) == 0 or req.max_new_tokens <= 0:
            raise ValueError("prompt and max_new_tokens must be positive")
        if self._reserve_tokens(req) > self.kv_capacity:
            raise ValueError(f"request needs {self._reserve_tokens(req)} KV tokens, capacity "
                             f"{self.kv_capacity}")
        req.admitted_iteration = self.iteration
        self.waiting.append(req)

    def _reserve_tokens(self, req: SeqRequest) -> int:
        total = len(req.prompt) + req.max_new_tokens
        return ((total + self.page - 1) // self.page) * self.page

    @property
    def reserved_tokens(self) -> int:
        return sum(self._reserve_tokens(r) for r in self.running.values())

    def has_work(self) -> bool:
        return bool(self.waiting) or any(not r.finished for r in self.running.values())

    # ------------------------------------------------------------ iteration
    def next_iteration(self) -> Iteration:
        t0 = time.perf_counter_ns()
        self.iteration += 1
        it = self.iteration
        runnable = [r for r in self.running.values() if r.prefill_complete and not r.finished]
        runnable.sort(key=lambda r: (r.last_served_iteration, r.admitted_ns, r.request_id))
        partial = [r for r in self.running.values() if not r.prefill_complete]
        starved = tuple(r.request_id for r in self.waiting
                        if it - r.admitted_iteration > self.starvation_limit)
        starved += tuple(r.request_id for r in runnable
                         if r.last_served_iteration >= 0 and it - r.last_served_iteration > self.starvation_limit)

        decode = runnable[: self.max_batch]
        if self.policy == SchedulerPolicy.THROUGHPUT and (self.waiting or partial):
            decode = []  # fill the batch first
        budget = self.budget
        allow_prefill = (not decode or self.policy != SchedulerPolicy.LATENCY or bool(starved))
        prefill: list[tuple[SeqRequest, int]] = []
        if allow_prefill:
            slots = self.max_batch - len(decode)
            # Continue partially prefilled prompts first, then admit new ones.
            for r in partial:
                if budget <= 0 or len(prefill) >= slots:
                    break
                n = min(budget, r.remaining_prompt)
                prefill.append((r, n))
                budget -= n
            while self.waiting and budget > 0 and len(prefill) < slots:
                cand = self.waiting[0]
                if self.reserved_tokens + self._reserve_tokens(cand) > self.kv_capacity:
                    break
                self.waiting.popleft()
                self.running[cand.request_id] = cand
                n = min(budget, cand.remaining_prompt)
                prefill.append((cand, n))
                budget -= n
        overhead = (time.perf_counter_ns() - t0) / 1e6
        now = time.monotonic_ns()
        waits = [(now - r.admitted_ns) / 1e6 for r in self.waiting]
        m = self.metrics
        m.iterations += 1
        m.overhead_ms += overhead
        m.batch_size_distribution[len(decode)] += 1
        for _, n in prefill:
            m.prefill_chunk_distribution[n] += 1
        m.starvation_events += len(starved)
        m.maximum_wait_ms = max(m.maximum_wait_ms, max(waits, default=0.0))
        return Iteration(it, tuple(r.request_id for r in decode),
                         tuple((r.request_id, n) for r, n in prefill), starved, overhead)

    # ------------------------------------------------------------ feedback
    def mark_prefill(self, request_id: str, tokens: int, sampled: int | None) -> None:
        r = self.running[request_id]
        r.prompt_consumed = min(len(r.prompt), r.prompt_consumed + tokens)
        r.last_served_iteration = self.iteration
        self.metrics.useful_tokens += tokens
        if r.prefill_complete and sampled is not None:
            self._append(r, sampled)

    def mark_decode(self, request_id: str, token: int) -> None:
        r = self.running[request_id]
        if not r.prefill_complete:
            raise ValueError(f"cannot decode {request_id!r} before its prefill completes")
        r.last_served_iteration = self.iteration
        self.metrics.useful_tokens += 1
        self._append(r, token)

    def _append(self, r: SeqRequest, token: int) -> None:
        if not r.output:
            r.first_token_ns = time.monotonic_ns()
        r.output.append(int(token))
        if len(r.output) >= r.max_new_tokens or int(token) in r.stop_token_ids:
            r.finished = True
            r.finish_ns = time.monotonic_ns()

    def pop_finished(self) -> list[SeqRequest]:
        done = [r for r in self.running.values() if r.finished]
        for r in done:
            del self.running[r.request_id]
        return done

    def cancel(self, request_id: str) -> SeqRequest | None:
        r = self.running.pop(request_id, None)
        if r is None:
            for w in list(self.waiting):
                if w.request_id == request_id:
                    self.waiting.remove(w)
                    return w
        return r

    def state(self) -> dict[str, Any]:
        return {
            "policy": self.policy.value,
            "iteration": self.iteration,
            "running": sorted(self.running),
            "waiting": [r.request_id for r in self.waiting],
            "kv_capacity_tokens": self.kv_capacity,
            "reserved_tokens": self.reserved_tokens,
            "metrics": self.metrics.payload(),
        }
