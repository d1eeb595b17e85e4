"""Pipeline stages x expert parallel serving of a MoE decoder on one box.

Ranks form a ``pp x ep`` grid: stage ``s = rank // ep`` owns a contiguous layer
interval (plus the embedding on stage 0, norm and LM head on the last stage);
inside a stage the ``ep`` ranks shard attention heads (tensor parallel, tokens
replicated) and experts (expert parallel) and reduce over an NCCL subgroup.
Stage boundaries move ``[micro-batch, hidden]`` bf16 activations with NCCL p2p
between the ranks of equal position in consecutive stages; each decode step
splits the batch into micro-batches so stage s works on micro-batch m while
stage s+1 works on m-1 (``parallel/pipeline.py``).  The last stage's greedy
tokens travel back to stage 0 for the next step.

``run_pp_bench`` is the benchmark entry used by ``bench.py --pp``: prefill
(TTFT) and device-timed decode steps, max over ranks.

Reference: the contiguous stage ring of si/worker/stage_runtime.py:2137-2275
(serial, TCP) -- here the stages are NCCL p2p peers on NVLink with micro-batch
overlap, and each stage is itself an EP group.
"""
from __future__ import annotations

import statistics

import torch
import torch.distributed as dist

from ..engine.kv_cache import PAGE, PagedKVCache
from ..models.config import ModelConfig
from ..models.dense import ForwardBatch, TPInfo
from ..models.moe import MoEModel, MoEWeights
from ..ops import attention as attn_ops
from .comm import NcclComm
from .pipeline import PipeGroup, PipelineStage, split_batch


def equal_layer_ranges(num_layers: int, num_stages: int) -> list[tuple[int, int]]:
    base, rem = divmod(num_layers, num_stages)
    out, s = [], 0
    for i in range(num_stages):
        n = base + (1 if i < rem else 0)
        out.append((s, s + n))
        s += n
    return out


class PPMoERank:
    """One rank of the pp x ep grid with its stage model, paged KV and micro-batch metadata."""

    def __init__(self, cfg: ModelConfig, pp: int, *, batch: int, max_seq: int, micro_batches: int,
                 device, seed: int = 0, comm: str = "nccl"):
        rank, world = dist.get_rank(), dist.get_world_size()
        if world % pp:
            raise ValueError(f"world {world} not divisible by pp {pp}")
        ep = world // pp
        self.stage, self.ep_rank = rank // ep, rank % ep
        self.pp, self.ep = pp, ep
        self.device = torch.device(device)
        # subgroups (every rank creates every group, in the same order)
        self.ep_group = None
        for s in range(pp):
            g = dist.new_group(list(range(s * ep, (s + 1) * ep)))
            if s == self.stage:
                self.ep_group = g
        self.pp_group = None
        for r in range(ep):
            g = dist.new_group([s * ep + r for s in range(pp)])
            if r == self.ep_rank:
                self.pp_group = g
        lo, hi = equal_layer_ranges(cfg.num_layers, pp)[self.stage]
        self.first, self.last = self.stage == 0, self.stage == pp - 1
        tp = TPInfo(self.ep_rank, ep)
        w = MoEWeights.random(cfg, tp, self.device, seed=seed, layer_range=(lo, hi),
                              with_embed=self.first, with_head=self.last)
        self.comm = NcclComm(self.ep_group) if ep > 1 else None
        self.comm_kind = "nccl" if ep > 1 else "none"
        if ep > 1 and comm == "ll":
            # The EP group's two reductions per layer (attention output, expert combine) go
            # through the low-latency NVLink all-reduce for decode micro-batches; prefill-sized
            # ones fall back to NCCL.
            from .ll_tp import LLTPComm
            self.comm = LLTPComm(self.comm, self.device, max_tokens=128, hidden=cfg.hidden_size)
            self.comm_kind = "ll_allreduce (attention output + expert combine) + nccl (prefill)"
        self.model = MoEModel(w, self.device, comm=self.comm, max_positions=max_seq + PAGE)
        self.cfg = cfg
        self.batch = batch
        self.mb_sizes = split_batch(batch, micro_batches)
        pages_per_seq = (max_seq + PAGE - 1) // PAGE
        self.max_pages = pages_per_seq
        self.kv = PagedKVCache(self.model.num_layers, self.model.num_kv_local, batch * pages_per_seq + 8,
                               self.device)
        self.bt = torch.arange(batch * pages_per_seq, dtype=torch.int32,
                               device=self.device).view(batch, pages_per_seq)
        self.pg = PipeGroup(self.stage, pp, [s * ep + self.ep_rank for s in range(pp)], self.pp_group)
        self.sm = torch.cuda.get_device_properties(self.device).multi_processor_count

    # ------------------------------------------------------------ batches
    def _mb_range(self, m: int) -> tuple[int, int]:
        s = sum(self.mb_sizes[:m])
        return s, s + self.mb_sizes[m]

    def decode_fb(self, m: int, ids: torch.Tensor, pos: int) -> ForwardBatch:
        a, b = self._mb_range(m)
        n = b - a
        bt = self.bt[a:b]
        p = torch.full((n,), pos, dtype=torch.int32, device=self.device)
        slots = (bt[:, pos // PAGE] * PAGE + pos % PAGE).to(torch.int32)
        return ForwardBatch(ids=ids, positions=p, slots=slots,
                            seq_lens=torch.full((n,), pos + 1, dtype=torch.int32, device=self.device),
                            block_table=bt, last_idx=torch.arange(n, device=self.device), is_decode=True,
                            decode_splits=attn_ops.decode_splits(n, self.model.num_kv_local,
                                                                 self.max_pages, self.sm))

    def prefill_fb(self, m: int, ids: torch.Tensor, P: int) -> ForwardBatch:
        a, b = self._mb_range(m)
        n = b - a
        bt = self.bt[a:b]
        pos = torch.arange(P, dtype=torch.int32, device=self.device).repeat(n)
        slots = (bt[:, :1] * PAGE).repeat(1, P).reshape(-1) + pos   # pages are contiguous per sequence
        return ForwardBatch(ids=ids, positions=pos, slots=slots.to(torch.int32),
                            seq_lens=torch.full((n,), P, dtype=torch.int32, device=self.device),
                            block_table=bt, last_idx=torch.arange(n, device=self.device) * P + P - 1,
                            is_decode=False,
                            cu_q=torch.arange(0, n * P + 1, P, dtype=torch.int32, device=self.device),
                            max_q_len=P)

    # ------------------------------------------------------------ steps
    def _stage_fn(self, fbs):
        def fn(m, x):
            fb = fbs[m]
            h = self.model.forward_hidden(fb, self.kv, h=None if self.first else x)
            if self.last:
                return self.model.greedy(self.model.logits(h, fb))
            return h
        return fn

    def step(self, fbs, inputs, rows_per_mb, rows_per_token: int = 1):
        """One pipelined pass; returns each micro-batch's greedy tokens on stage 0."""
        st = PipelineStage(self.pg, self._stage_fn(fbs), self.cfg.hidden_size, device=self.device)
        st.result_shape = lambda rows: (rows // rows_per_token,)
        return st.step(inputs, rows_per_mb)


def run_pp_bench(args, cfg: ModelConfig, rank: int, world: int, local: int) -> dict:
    from ..utils.timing import ClockSampler
    pp = args.pp
    B, P, K, W = args.batch, args.prompt_len, args.steps, args.warmup
    M = max(1, args.micro_batches)
    dev = torch.device("cuda", local)
    comm = getattr(args, "comm", "nccl")
    r = PPMoERank(cfg, pp, batch=B, max_seq=P + K + W + 8, micro_batches=M, device=dev,
                  comm="ll" if comm in ("ll", "auto") else "nccl")
    g = torch.Generator().manual_seed(0)
    prompts = torch.randint(0, cfg.vocab_size, (B, P), generator=g)

    def barrier():
        dist.barrier()
        torch.cuda.synchronize()

    # prefill: per micro-batch, whole prompts through the pipeline
    fbs = []
    inputs = []
    for m in range(len(r.mb_sizes)):
        a, b = r._mb_range(m)
        ids = prompts[a:b].reshape(-1).to(dev)
        fbs.append(r.prefill_fb(m, ids, P))
        inputs.append(ids)
    rows = [n * P for n in r.mb_sizes]
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    toks = r.step(fbs, inputs if r.first else None, rows, rows_per_token=P)
    e1.record()
    barrier()
    ttft = _max(e0.elapsed_time(e1), dev)
    # decode: tokens live on stage 0 (returned by the last stage); other stages get hidden states
    cur = toks if r.first else [torch.zeros(n, dtype=torch.int64, device=dev) for n in r.mb_sizes]
    pos = P

    def decode_step(cur, pos):
        fbs = [r.decode_fb(m, cur[m], pos) for m in range(len(r.mb_sizes))]
        out = r.step(fbs, cur if r.first else None, list(r.mb_sizes))
        return out if r.first else cur

    for _ in range(W):
        cur = decode_step(cur, pos)
        pos += 1
    barrier()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(K + 1)]
    with ClockSampler(local) as clocks:
        evs[0].record()
        for i in range(K):
            cur = decode_step(cur, pos)
            pos += 1
            evs[i + 1].record()
        barrier()
    total = _max(evs[0].elapsed_time(evs[-1]), dev)
    tpot = _max(statistics.median(evs[i].elapsed_time(evs[i + 1]) for i in range(K)), dev)
    clk = clocks.summary()
    value = B * K / (total / 1e3)
    return {
        "metric": args.metric, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": total / K, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (uniform random token ids, random N(0,0.02) weights)",
        "config": {"model": cfg.name, "global_batch": B, "seq_len": P, "decode_tokens": K,
                   "parallelism": f"pp{pp}x(tp{world // pp}-attention+ep{world // pp})",
                   "micro_batches": len(r.mb_sizes), "stage_boundary": "nccl p2p, micro-batch overlap",
                   "comm": r.comm_kind,
                   "l2": "weights per stage exceed L2; no flush needed"},
        "ttft_ms_p50": ttft, "tpot_ms_p50": tpot,
        "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"], "reasons": clk["reasons"]},
        "e2e": None, "gpu_launches": None, "impl": "ours",
    }


def _max(x: float, dev) -> float:
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
