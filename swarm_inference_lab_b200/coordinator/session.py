"""Coordinator-side session control over a stage ring, with restart-and-replay.

Per request: open the session on the ring (stage 0 forwards it down),
prefill the prompt, then drive one DECODE per output token into stage 0 and
accept the TOKEN_RESULT it relays back.  Hidden states only flow stage to
stage; the coordinator sees token ids (and, in verification mode, the last
stage's logits).

On a transport failure the controller asks its ``recover`` callback for a
(possibly new) route generation, opens a fresh session, replays the prompt
and every accepted token exactly as they were first computed, checks that
the replay reproduces each accepted token (any divergence fails closed with
:class:`IntegrityError`), and resumes at the first unaccepted position.

Reference: si/coordinator/session_controller.py:99-1289 (token loop :236-263,
_recover :926, replay :1006-1035).
"""
from __future__ import annotations

import time
import uuid
from dataclasses import dataclass, field
from typing import Awaitable, Callable

import torch

from ..engine.speculative import prompt_lookup_draft
from ..protocol import stage_ring as sr
from ..transport.stage_ring_net import ConnectionPool, TransportError
from ..transport.tensor_codec import pack_tensor, unpack_tensor


class IntegrityError(RuntimeError):
    """A replay produced a token different from one already accepted."""


class StageError(RuntimeError):
    """A stage answered with an ERROR frame."""


@dataclass
class Route:
    stage0: tuple[str, int]
    generation: int
    topology_id: str
    model_revision: str
    stage0_layers: tuple[int, int]
    tokenizer_revision: str = "none"


@dataclass
class SessionResult:
    request_id: str
    tokens: list[int]
    logits: list[torch.Tensor] = field(default_factory=list)
    recoveries: int = 0
    generations: list[int] = field(default_factory=list)
    ttft_ms: float = 0.0
    total_ms: float = 0.0

    @property
    def tpot_ms(self) -> float:
        n = len(self.tokens)
        return (self.total_ms - self.ttft_ms) / max(1, n - 1)


Recover = Callable[[Route, Exception], Awaitable[Route]]


class SessionController:
    def __init__(self, route: Route, *, pool: ConnectionPool | None = None,
                 recover: Recover | None = None, max_recoveries: int = 3,
                 return_logits: bool = False, speculate_k: int = 0,
                 spec_min_accept: float = 0.1, spec_warmup: int = 8):
        self.route = route
        self.pool = pool or ConnectionPool()
        self.recover_cb = recover
        self.max_recoveries = max_recoveries
        self.return_logits = return_logits
        # Exact speculation (off by default): up to ``speculate_k`` prompt-lookup draft tokens
        # are verified in one VERIFY_CANDIDATES pass through the ring; the longest prefix that
        # equals the greedy predictions is accepted plus one token, so the output is exactly
        # the greedy output.  Not combined with per-token logits.
        # Drafting stops for the rest of a stream once, after ``spec_warmup`` verifications,
        # fewer than ``spec_min_accept`` of the drafted tokens were accepted (a verification
        # that rarely pays costs a frame per token like plain decode, with bigger frames).
        self.speculate_k = 0 if return_logits else int(speculate_k)
        self.spec_min_accept = spec_min_accept
        self.spec_warmup = spec_warmup
        self.spec_stats = {"verify_calls": 0, "drafted": 0, "accepted": 0, "disabled": False}
        self.seq = sr.SequenceAllocator()
        self.events: list[dict] = []

    def _msg(self, op, session_id, request_id, position, payload=b"", attrs=None, shape=(),
             dtype="none") -> sr.StageMessage:
        r = self.route
        a = dict(attrs or {})
        a["generation"] = r.generation
        return sr.StageMessage(
            operation=op, model_revision=r.model_revision, tokenizer_revision=r.tokenizer_revision,
            topology_id=r.topology_id, stage_id=0, layer_start=r.stage0_layers[0],
            layer_end=r.stage0_layers[1], session_id=session_id, request_id=request_id,
            sequence_number=self.seq.next(session_id, sr.COORDINATOR, 0)
            if op not in (sr.Operation.OPEN_SESSION, sr.Operation.HEALTH) else 0,
            token_position=position, source_stage=sr.COORDINATOR, destination_stage=0,
            tensor_shape=tuple(shape), tensor_dtype=dtype, payload=payload, attributes=a)

    async def _call(self, msg) -> sr.StageMessage:
        rep = await self.pool.send(*self.route.stage0, msg)
        if rep.operation == sr.Operation.ERROR:
            raise StageError(f"{rep.attributes.get('error')}: {rep.attributes.get('detail')}")
        return rep

    async def _run_tokens(self, session_id, request_id, ids: list[int], position: int,
                          op: sr.Operation, replay: bool,
                          truncate_to: int | None = None) -> tuple[int, torch.Tensor | None]:
        pk = pack_tensor(torch.tensor(ids, dtype=torch.int64))
        attrs = {"tensor": pk.attributes, "replay": replay}
        if truncate_to is not None:
            attrs["truncate_to"] = int(truncate_to)
        if self.return_logits:
            attrs["return_logits"] = True
        rep = await self._call(self._msg(op, session_id, request_id, position, pk.payload, attrs,
                                         pk.shape, "int64"))
        logits = None
        if rep.payload and "tensor" in rep.attributes:
            logits = unpack_tensor(rep.payload, rep.attributes["tensor"])
        return int(rep.attributes["token"]), logits

    async def _verify(self, session_id, request_id, ids: list[int], position: int,
                      truncate_to: int | None) -> list[int]:
        """One VERIFY_CANDIDATES pass of ``ids`` (the last accepted token then the draft) at
        ``position``: the greedy token after every row."""
        pk = pack_tensor(torch.tensor(ids, dtype=torch.int64))
        attrs = {"tensor": pk.attributes, "replay": False}
        if truncate_to is not None:
            attrs["truncate_to"] = int(truncate_to)
        rep = await self._call(self._msg(sr.Operation.VERIFY_CANDIDATES, session_id, request_id,
                                         position, pk.payload, attrs, pk.shape, "int64"))
        return [int(t) for t in rep.attributes["tokens"]]

    async def _open(self, session_id, request_id):
        await self._call(self._msg(sr.Operation.OPEN_SESSION, session_id, request_id, -1))

    async def _close(self, session_id, request_id, cancel=False):
        op = sr.Operation.CANCEL_SESSION if cancel else sr.Operation.CLOSE_SESSION
        try:
            await self._call(self._msg(op, session_id, request_id, -1))
        except (TransportError, StageError):
            pass
        self.seq.reset_session(session_id)

    async def generate(self, prompt: list[int], max_new_tokens: int,
                       request_id: str | None = None) -> SessionResult:
        """Runs the request to completion (see :meth:`stream`)."""
        request_id = request_id or uuid.uuid4().hex[:12]
        res = SessionResult(request_id, [])
        t_start = time.perf_counter()
        async for ev in self.stream(prompt, max_new_tokens, request_id):
            if ev["event"] == "token":
                res.tokens.append(ev["token"])
                res.logits.append(ev["logits"])
                if ev["index"] == 0:
                    res.ttft_ms = (time.perf_counter() - t_start) * 1e3
            elif ev["event"] == "recovered":
                res.recoveries += 1
            if ev["event"] in ("started", "recovered"):
                res.generations.append(ev["generation"])
        res.total_ms = (time.perf_counter() - t_start) * 1e3
        return res

    async def stream(self, prompt: list[int], max_new_tokens: int, request_id: str | None = None):
        """Async generator of the request's events: ``started`` (route generation), one
        ``token`` per accepted output token (index, token, logits or None) and ``recovered``
        (new generation) after a restart-and-replay.  The next token is computed only when
        the consumer asks for the next event, so a consumer paces the decode."""
        request_id = request_id or uuid.uuid4().hex[:12]
        tokens: list[int] = []
        recoveries = 0
        session_id = f"{request_id}:g{self.route.generation}"
        self.current = (session_id, request_id)
        yield {"event": "started", "request": request_id, "generation": self.route.generation}
        need_open = True
        recovering = False
        while True:
            try:
                if need_open:
                    await self._open(session_id, request_id)
                    need_open = False
                    # (Re)build the session: prompt, then each accepted token one by one.
                    tok, lg = await self._run_tokens(session_id, request_id, prompt, 0,
                                                     sr.Operation.PREFILL, replay=bool(tokens))
                    if recovering:
                        recovering = False
                        yield {"event": "recovered", "request": request_id,
                               "generation": self.route.generation, "replayed": len(tokens)}
                    if not tokens:
                        tokens.append(tok)
                        self.events.append({"event": "first_token", "request": request_id})
                        yield {"event": "token", "index": 0, "token": tok, "logits": lg}
                    else:
                        if tok != tokens[0]:
                            raise IntegrityError(f"replay diverged at output 0: {tok} != {tokens[0]}")
                        for i in range(len(tokens) - 1):
                            t2, _ = await self._run_tokens(session_id, request_id, [tokens[i]],
                                                           len(prompt) + i, sr.Operation.DECODE, True)
                            if t2 != tokens[i + 1]:
                                raise IntegrityError(
                                    f"replay diverged at output {i + 1}: {t2} != {tokens[i + 1]}")
                        self.events.append({"event": "replay_complete", "request": request_id,
                                            "tokens": len(tokens)})
                # Cache length the stages must roll back to before the next frame (rejected
                # candidates of the last verification), or None.
                trunc = None
                calls0, drafted0, accepted0 = (self.spec_stats["verify_calls"],
                                               self.spec_stats["drafted"], self.spec_stats["accepted"])
                drafting = bool(self.speculate_k)
                while len(tokens) < max_new_tokens:
                    pos = len(prompt) + len(tokens) - 1
                    draft = []
                    if drafting:
                        draft = prompt_lookup_draft(prompt + tokens, self.speculate_k)
                        draft = draft[:max(0, max_new_tokens - len(tokens) - 1)]
                    if draft:
                        preds = await self._verify(session_id, request_id, [tokens[-1]] + draft,
                                                   pos, trunc)
                        m = 0
                        while m < len(draft) and draft[m] == preds[m]:
                            m += 1
                        trunc = pos + 1 + m if m < len(draft) else None
                        self.spec_stats["verify_calls"] += 1
                        self.spec_stats["drafted"] += len(draft)
                        self.spec_stats["accepted"] += m
                        calls = self.spec_stats["verify_calls"] - calls0
                        drafted = self.spec_stats["drafted"] - drafted0
                        accepted = self.spec_stats["accepted"] - accepted0
                        if calls >= self.spec_warmup and accepted < self.spec_min_accept * drafted:
                            drafting = False
                            self.spec_stats["disabled"] = True
                        for tok in preds[:m + 1]:
                            tokens.append(tok)
                            yield {"event": "token", "index": len(tokens) - 1, "token": tok,
                                   "logits": None}
                        continue
                    tok, lg = await self._run_tokens(session_id, request_id, [tokens[-1]], pos,
                                                     sr.Operation.DECODE, False, trunc)
                    trunc = None
                    tokens.append(tok)
                    yield {"event": "token", "index": len(tokens) - 1, "token": tok, "logits": lg}
                break
            except (TransportError, StageError) as exc:
                if isinstance(exc, StageError) and "IntegrityError" in str(exc):
                    raise
                recoveries += 1
                self.events.append({"event": "recovery_started", "request": request_id,
                                    "error": str(exc), "accepted": len(tokens)})
                if recoveries > self.max_recoveries or self.recover_cb is None:
                    raise
                await self._close(session_id, request_id, cancel=True)
                self.route = await self.recover_cb(self.route, exc)
                session_id = f"{request_id}:g{self.route.generation}:r{recoveries}"
                self.current = (session_id, request_id)
                need_open = True
                recovering = True
        await self._close(session_id, request_id)
        self.current = None

    async def cancel_current(self, *, finished: bool = False) -> bool:
        """Ends the session of the stream this controller ran last, on every stage (for a
        consumer that stopped reading the stream before its end): a cancel, or with
        ``finished`` an ordinary close (the request ended early, e.g. on a stop token).
        False if none is open."""
        if getattr(self, "current", None) is None:
            return False
        session_id, request_id = self.current
        self.current = None
        await self._close(session_id, request_id, cancel=not finished)
        return True
