"""Universal worker ABI: backend-neutral jobs (generate, draft, verify, background) and a
bounded asynchronous execution queue.

Jobs are plain JSON-compatible records so any backend (this runtime's engine, an
external engine, a test double) can serve them:

    generate   {prompt, max_new_tokens}                     -> {tokens}
    draft      {context, k}                                 -> {draft}        (proposals)
    verify     {context, candidates}                        -> {accepted, next}
    background {name, args}                                 -> {result}       (maintenance)

``UniversalWorker`` validates a job, dispatches it to the backend's method of the same
name and wraps the result with timing; unknown kinds and malformed jobs are rejected
with an error record instead of an exception.  ``ExecutionQueue`` admits at most
``max_pending`` jobs, runs up to ``concurrency`` at a time, and batches consecutive
jobs of one kind into a single backend call when the backend offers ``<kind>_batch``.

Reference: si/worker/abi.py:106-300 (job ABI), si/worker/universal.py:85,276,
si/worker/execution.py:37 (bounded queue with nominal batching).
"""
from __future__ import annotations

import asyncio
import time
from dataclasses import dataclass, field

JOB_FIELDS = {
    "generate": ("prompt", "max_new_tokens"),
    "draft": ("context", "k"),
    "verify": ("context", "candidates"),
    "background": ("name",),
}


class JobError(ValueError):
    pass


def validate_job(job: dict) -> str:
    kind = job.get("kind")
    if kind not in JOB_FIELDS:
        raise JobError(f"unknown job kind {kind!r}")
    missing = [f for f in JOB_FIELDS[kind] if f not in job]
    if missing:
        raise JobError(f"{kind} job lacks {missing}")
    if kind == "generate" and (not isinstance(job["prompt"], list) or int(job["max_new_tokens"]) < 0):
        raise JobError("generate: prompt must be a token list and max_new_tokens >= 0")
    if kind == "verify" and not isinstance(job["candidates"], list):
        raise JobError("verify: candidates must be a token list")
    return kind


class GreedyVerifier:
    """Reference semantics of ``verify`` for any greedy ``next_token(context)`` backend:
    accept the longest candidate prefix the backend itself would have produced."""

    def __init__(self, next_token):
        self.next_token = next_token

    def verify(self, context: list[int], candidates: list[int]) -> dict:
        ctx = list(context)
        accepted = 0
        for c in candidates:
            t = self.next_token(ctx)
            if t != c:
                return {"accepted": accepted, "next": t}
            ctx.append(c)
            accepted += 1
        return {"accepted": accepted, "next": self.next_token(ctx)}


class UniversalWorker:
    def __init__(self, backend, worker_id: str = "worker"):
        self.backend = backend
        self.worker_id = worker_id

    def run(self, job: dict) -> dict:
        t0 = time.perf_counter()
        try:
            kind = validate_job(job)
            fn = getattr(self.backend, kind, None)
            if fn is None:
                raise JobError(f"backend does not serve {kind} jobs")
            args = {k: v for k, v in job.items() if k not in ("kind", "job_id")}
            result = fn(**args)
            status = "OK"
        except JobError as exc:
            result, status = {"error": str(exc)}, "REJECTED"
        except Exception as exc:  # noqa: BLE001 - a backend failure becomes the job's result
            result, status = {"error": f"{type(exc).__name__}: {exc}"}, "ERROR"
        return {"job_id": job.get("job_id"), "worker": self.worker_id, "status": status,
                "ms": (time.perf_counter() - t0) * 1e3, **({"result": result})}


@dataclass
class ExecutionQueue:
    worker: UniversalWorker
    max_pending: int = 64
    concurrency: int = 1
    max_batch: int = 8
    _q: asyncio.Queue | None = None
    _tasks: list = field(default_factory=list)
    stats: dict = field(default_factory=lambda: {"submitted": 0, "rejected": 0, "batches": 0})

    async def start(self):
        self._q = asyncio.Queue(self.max_pending)
        self._tasks = [asyncio.create_task(self._loop()) for _ in range(self.concurrency)]

    async def submit(self, job: dict) -> dict:
        if self._q.full():
            self.stats["rejected"] += 1
            return {"job_id": job.get("job_id"), "status": "REJECTED", "result": {"error": "queue full"}}
        fut = asyncio.get_running_loop().create_future()
        self._q.put_nowait((job, fut))
        self.stats["submitted"] += 1
        return await fut

    async def _loop(self):
        while True:
            job, fut = await self._q.get()
            batch = [(job, fut)]
            kind = job.get("kind")
            batch_fn = getattr(self.worker.backend, f"{kind}_batch", None)
            while batch_fn is not None and len(batch) < self.max_batch and not self._q.empty():
                nxt = self._q._queue[0]  # peek: only same-kind jobs join the batch
                if nxt[0].get("kind") != kind:
                    break
                batch.append(self._q.get_nowait())
            self.stats["batches"] += 1
            if batch_fn is not None and len(batch) > 1:
                try:
                    kinds = [validate_job(j) for j, _ in batch]
                    assert all(k == kind for k in kinds)
                    results = await asyncio.to_thread(
                        batch_fn, [{k: v for k, v in j.items() if k not in ("kind", "job_id")} for j, _ in batch])
                    for (j, f), r in zip(batch, results):
                        f.set_result({"job_id": j.get("job_id"), "worker": self.worker.worker_id,
                                      "status": "OK", "result": r})
                except Exception as exc:  # noqa: BLE001
                    for j, f in batch:
                        f.set_result({"job_id": j.get("job_id"), "status": "ERROR",
                                      "result": {"error": str(exc)}})
            else:
                for j, f in batch:
                    f.set_result(await asyncio.to_thread(self.worker.run, j))

    async def close(self):
        for t in self._tasks:
            t.cancel()
        await asyncio.gather(*self._tasks, return_exceptions=True)
