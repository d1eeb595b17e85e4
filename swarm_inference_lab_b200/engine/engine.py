"""Public serving API of one stage owner: ``LLMEngine``.

``LLMEngine`` owns the model weights, the resident paged KV cache, the
continuous-batching scheduler and the CUDA-graph decode runner of one rank
(or of every rank of a tensor-parallel group, each process holding its
shard).  ``generate`` runs requests to completion and reports the serving
metrics the benchmark quotes (decode tokens/s, p50 TTFT and TPOT); ``step``
runs one scheduler iteration for callers that stream.

Counterpart of the reference's single-process fast engine
(si/model/qwen3_engine.py:387 ``Qwen3FastEngine``, :691 ``generate_batch``).
"""
from __future__ import annotations

import itertools
import statistics
import time
from dataclasses import dataclass, field

import torch

from ..models.config import ModelConfig
from ..models.deepseek import MLAModel, MLAWeights
from ..models.dense import DenseModel, DenseWeights, TPInfo
from ..models.moe import MoEModel, MoEWeights
from .kv_cache import PAGE, PagedKVCache
from .runner import ModelRunner, bucket_for
from .scheduler import ContinuousScheduler, SchedulerPolicy, SeqRequest


@dataclass
class SamplingParams:
    """Per-request decoding options.  ``temperature`` 0 selects greedy decoding (lowest
    id on ties).  Otherwise the repetition penalty (over prompt + output), temperature,
    top-k and top-p (nucleus) shape the distribution and a Gumbel-max draw from a Philox
    stream keyed by ``seed`` (a hash of the request id when None) and the token index picks
    the token, inside the captured decode graph."""
    max_new_tokens: int = 16
    temperature: float = 0.0
    top_k: int = 0
    top_p: float = 1.0
    repetition_penalty: float = 1.0
    seed: int | None = None
    stop_token_ids: tuple[int, ...] = ()

    @property
    def greedy(self) -> bool:
        return self.temperature == 0.0 and self.repetition_penalty == 1.0


@dataclass
class RequestOutput:
    request_id: str
    prompt_len: int
    token_ids: list[int]
    ttft_ms: float
    tpot_ms: float


@dataclass
class GenerationMetrics:
    requests: int
    output_tokens: int
    prefill_ms: float
    decode_ms: float
    decode_steps: int
    decode_tokens_per_s: float
    ttft_ms_p50: float
    tpot_ms_p50: float
    step_ms: list[float] = field(default_factory=list)


class LLMEngine:
    def __init__(self, cfg: ModelConfig, *, device: str | torch.device = "cuda",
                 weights: DenseWeights | None = None, seed: int = 0, comm=None,
                 tp: TPInfo | None = None, max_batch: int = 64, max_seq_len: int = 4096,
                 kv_pages: int | None = None, prefill_token_budget: int = 16384,
                 policy: str = SchedulerPolicy.BALANCED, use_cuda_graphs: bool = True):
        self.cfg = cfg
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.tp = tp or TPInfo()
        max_pos = max(max_seq_len, 1) + PAGE
        if kv_pages is None:
            kv_pages = max_batch * ((max_seq_len + PAGE - 1) // PAGE) + 8
        if cfg.mla:
            # MLA: data-parallel attention with a latent cache; ``tp`` is the expert-parallel group.
            self.weights = weights or MLAWeights.random(cfg, self.tp, self.device, seed=seed)
            self.model = MLAModel(self.weights, self.device, comm=comm, max_positions=max_pos)
            self.kv = PagedKVCache(self.model.num_layers, 1, kv_pages, self.device,
                                   latent_dim=self.model.latent_dim)
        else:
            if cfg.is_moe:
                self.weights = weights or MoEWeights.random(cfg, self.tp, self.device, seed=seed)
                self.model = MoEModel(self.weights, self.device, comm=comm, max_positions=max_pos)
            else:
                self.weights = weights or DenseWeights.random(cfg, self.tp, self.device, seed=seed)
                self.model = DenseModel(self.weights, self.device, comm=comm, max_positions=max_pos)
            self.kv = PagedKVCache(self.model.num_layers, self.model.num_kv_local, kv_pages,
                                   self.device)
        self.runner = ModelRunner(self.model, self.kv, max_seq_len=max_seq_len,
                                  use_cuda_graphs=use_cuda_graphs)
        self.max_batch = max_batch
        self.max_seq_len = max_seq_len
        self.scheduler = ContinuousScheduler(max_batch=max_batch,
                                             prefill_token_budget=prefill_token_budget,
                                             kv_capacity_tokens=kv_pages * PAGE, policy=policy)
        self._ids = itertools.count()
        self._finished: dict[str, SeqRequest] = {}

    # ------------------------------------------------------------ requests
    def add_request(self, prompt: list[int], params: SamplingParams | None = None,
                    request_id: str | None = None) -> str:
        params = params or SamplingParams()
        if params.temperature < 0 or params.top_p <= 0 or params.top_p > 1 or params.top_k < 0:
            raise ValueError("temperature >= 0, 0 < top_p <= 1 and top_k >= 0 are required")
        if params.repetition_penalty <= 0:
            raise ValueError("repetition_penalty must be positive")
        rid = request_id or f"req-{next(self._ids)}"
        if len(prompt) + params.max_new_tokens > self.max_seq_len:
            raise ValueError("prompt + max_new_tokens exceeds max_seq_len")
        sampling = None
        if not params.greedy:
            import hashlib
            seed = params.seed if params.seed is not None else int.from_bytes(
                hashlib.sha256(rid.encode()).digest()[:7], "little")
            sampling = SamplingParams(**{**params.__dict__, "seed": int(seed)})
        self.scheduler.admit(SeqRequest(rid, list(prompt), params.max_new_tokens,
                                        time.monotonic_ns(), stop_token_ids=params.stop_token_ids,
                                        sampling=sampling))
        return rid

    def cancel(self, request_id: str) -> None:
        self.scheduler.cancel(request_id)
        self.kv.close(request_id)

    # ------------------------------------------------------------ iteration
    def step(self) -> list[tuple[str, int]]:
        """One continuous-batching iteration; returns the (request, token) pairs produced."""
        it = self.scheduler.next_iteration()
        produced: list[tuple[str, int]] = []
        sch = self.scheduler
        if it.prefill:
            ids, starts, pages, rids = [], [], [], []
            for rid, n in it.prefill:
                r = sch.running[rid]
                if rid not in self.kv.seqs:
                    self.kv.open(rid)
                    self.kv.reserve(rid, len(r.prompt) + r.max_new_tokens)
                ids.append(r.prompt[r.prompt_consumed:r.prompt_consumed + n])
                starts.append(r.prompt_consumed)
                pages.append(self.kv.seqs[rid].pages)
                rids.append((rid, n))
            samp = [sch.running[rid].sampling for rid, _ in rids]
            hist = [sch.running[rid].prompt for rid, _ in rids]
            toks = self.runner.prefill(ids, starts, pages,
                                       sampling=samp if any(samp) else None, history=hist).tolist()
            for (rid, n), t in zip(rids, toks):
                r = sch.running[rid]
                done = r.prompt_consumed + n >= len(r.prompt)
                sch.mark_prefill(rid, n, t if done else None)
                self.kv.seqs[rid].length = r.context_len
                if done:
                    produced.append((rid, t))
        if it.decode:
            reqs = [sch.running[rid] for rid in it.decode]
            ids = [r.output[-1] for r in reqs]
            positions = [r.context_len - 1 for r in reqs]
            pages = [self.kv.seqs[r.request_id].pages for r in reqs]
            samp = [r.sampling for r in reqs]
            if any(samp):
                toks = self.runner.decode(ids, positions, pages, sampling=samp,
                                          history=[r.prompt + r.output for r in reqs],
                                          steps=[len(r.output) for r in reqs])
            else:
                toks = self.runner.decode(ids, positions, pages)
            for r, t in zip(reqs, toks):
                sch.mark_decode(r.request_id, t)
                self.kv.seqs[r.request_id].length = r.context_len
                produced.append((r.request_id, t))
        for r in sch.pop_finished():
            self.kv.close(r.request_id)
            self._finished[r.request_id] = r
        return produced

    def generate(self, prompts: list[list[int]], params: SamplingParams | None = None
                 ) -> tuple[list[RequestOutput], GenerationMetrics]:
        """Serve ``prompts`` to completion; returns outputs in prompt order plus metrics."""
        params = params or SamplingParams()
        self._finished = {}
        rids = [self.add_request(p, params) for p in prompts]
        t_start = time.perf_counter()
        prefill_ms = decode_ms = 0.0
        steps = 0
        step_ms: list[float] = []
        while self.scheduler.has_work():
            had_prefill = bool(self.scheduler.waiting) or any(
                not r.prefill_complete for r in self.scheduler.running.values())
            t0 = time.perf_counter()
            self.step()
            dt = (time.perf_counter() - t0) * 1e3
            if had_prefill:
                prefill_ms += dt
            else:
                decode_ms += dt
                steps += 1
                step_ms.append(dt)
        _ = t_start
        outs = []
        for rid, p in zip(rids, prompts):
            r = self._finished[rid]
            ttft = (r.first_token_ns - r.admitted_ns) / 1e6
            n = len(r.output)
            tpot = (r.finish_ns - r.first_token_ns) / 1e6 / max(1, n - 1)
            outs.append(RequestOutput(rid, len(p), list(r.output), ttft, tpot))
        dec_tokens = sum(max(0, len(o.token_ids) - 1) for o in outs)
        m = GenerationMetrics(
            requests=len(outs), output_tokens=sum(len(o.token_ids) for o in outs),
            prefill_ms=prefill_ms, decode_ms=decode_ms, decode_steps=steps,
            decode_tokens_per_s=dec_tokens / (decode_ms / 1e3) if decode_ms > 0 else 0.0,
            ttft_ms_p50=statistics.median(o.ttft_ms for o in outs) if outs else 0.0,
            tpot_ms_p50=statistics.median(o.tpot_ms for o in outs) if outs else 0.0,
            step_ms=step_ms)
        return outs, m

    def warmup(self, batch_sizes=(1,)) -> None:
        for b in batch_sizes:
            self.runner.graph_for(bucket_for(b))
