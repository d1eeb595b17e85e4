"""Parallelism planner for one NVLink domain (e.g. 8x B200): picks TP / EP / PP / DP
splits by predicted decode throughput, TTFT and memory, from MEASURED box constants.

Model of one decode step on one rank (all terms reported by ``explain``):

    t_step = (W_rank + KV_rank) / (eta * HBM)              weight + KV streaming
           + launches * t_launch                           per-kernel fixed cost
           + n_allreduce * (alpha + beta * bytes_AR)       tensor/expert-parallel reduction
           + (pp - 1) * (lat_p2p + bytes_act / BW_nvlink)  pipeline boundaries

``eta`` and ``t_launch`` are fitted (least squares) to measured decode steps;
``alpha``/``beta`` to measured all-reduce latencies and ``BW_nvlink`` /
``lat_p2p`` come from the NVLink probe (``parallel/nvlink_probe.py``).
Unmeasured constants fall back to nominal values and cost the plan the
cost model's 0.98 penalty each.

Reference: the collective projection of si/microsharding/projection.py:23-601
(analytic steps/bytes per collective; its NVLink profile was a constant
0.01 ms / 400,000 Mbps) and the canonical plan scoring of si/engines/cost_model.py.
"""
from __future__ import annotations

import json
import math
from dataclasses import asdict, dataclass, field
from pathlib import Path

from ..models.config import ModelConfig
from .cost_model import PlanCostInputs, score_costs

GB = 1e9


@dataclass
class BoxMeasurements:
    hbm_gbs: float = 6534.1
    bf16_tflops: float = 1649.5
    gpu_memory_gb: float = 179.0
    nvlink_gbs: float = 770.0          # per direction, peer copy
    nvlink_latency_us: float = 3.0
    ar_alpha_us: float = 12.0          # all-reduce latency at tiny sizes
    ar_beta_us_per_mb: float = 2.6     # incremental cost per MB
    eta: float = 0.62                  # achieved fraction of HBM bandwidth in decode
    launch_us: float = 2.0             # fixed cost per kernel inside a graph
    measured: set = field(default_factory=set)

    @classmethod
    def from_files(cls, peaks: str | None = None, probe: str | None = None) -> "BoxMeasurements":
        m = cls()
        if peaks and Path(peaks).exists():
            d = json.loads(Path(peaks).read_text())
            m.hbm_gbs = float(d.get("hbm_gbs", m.hbm_gbs))
            m.bf16_tflops = float(d.get("bf16_tflops", m.bf16_tflops))
            m.measured |= {"hbm_gbs", "bf16_tflops"}
        if probe and Path(probe).exists():
            d = json.loads(Path(probe).read_text())
            for k in ("nvlink_gbs", "nvlink_latency_us", "ar_alpha_us", "ar_beta_us_per_mb", "eta",
                      "launch_us"):
                if k in d:
                    setattr(m, k, float(d[k]))
                    m.measured.add(k)
        return m

    def fit_decode(self, observations: list[tuple[float, int, float]]) -> None:
        """Fit eta and launch_us from (bytes streamed, kernel launches, measured ms) triples."""
        if len(observations) < 2:
            return
        # ms = bytes / (eta * HBM) + launches * launch_us  -> linear in (1/eta, launch_us)
        xs = [(b / (self.hbm_gbs * GB) * 1e3, n / 1e3, ms) for b, n, ms in observations]
        s11 = sum(a * a for a, _, _ in xs); s12 = sum(a * c for a, c, _ in xs)
        s22 = sum(c * c for _, c, _ in xs)
        t1 = sum(a * y for a, _, y in xs); t2 = sum(c * y for _, c, y in xs)
        det = s11 * s22 - s12 * s12
        if abs(det) < 1e-18:
            return
        inv_eta = (t1 * s22 - t2 * s12) / det
        launch = (s11 * t2 - s12 * t1) / det
        if inv_eta > 0:
            self.eta = min(1.0, 1.0 / inv_eta)
            self.launch_us = max(0.0, launch)
            self.measured |= {"eta", "launch_us"}

    def fit_allreduce(self, samples: list[tuple[int, float]]) -> None:
        """Fit alpha/beta from (bytes, microseconds) all-reduce samples."""
        if len(samples) < 2:
            return
        n = len(samples)
        xs = [b / 1e6 for b, _ in samples]
        ys = [us for _, us in samples]
        mx, my = sum(xs) / n, sum(ys) / n
        vx = sum((x - mx) ** 2 for x in xs)
        if vx <= 0:
            return
        beta = sum((x - mx) * (y - my) for x, y in zip(xs, ys)) / vx
        self.ar_beta_us_per_mb = max(0.0, beta)
        self.ar_alpha_us = max(0.0, my - beta * mx)
        self.measured |= {"ar_alpha_us", "ar_beta_us_per_mb"}


@dataclass
class BoxPlan:
    tp: int
    ep: int
    pp: int
    dp: int
    step_ms: float
    ttft_ms: float
    tokens_per_s: float
    memory_gb_per_gpu: float
    fits: bool
    score: float
    terms: dict


def _bytes_per_layer(cfg: ModelConfig, dtype_bytes: float = 2.0) -> tuple[float, float]:
    """(dense bytes per layer, expert bytes per layer) for the weights."""
    H = cfg.hidden_size
    if cfg.mla:
        qk = cfg.qk_nope_head_dim + cfg.qk_rope_head_dim
        attn = (H * cfg.q_lora_rank + cfg.q_lora_rank * cfg.num_heads * qk
                + H * (cfg.kv_lora_rank + cfg.qk_rope_head_dim)
                + cfg.kv_lora_rank * cfg.num_heads * (cfg.qk_nope_head_dim + cfg.v_head_dim)
                + cfg.num_heads * cfg.v_head_dim * H)
    else:
        attn = H * (cfg.q_size + 2 * cfg.kv_size) + cfg.q_size * H
    w_bytes = 1.0 if cfg.weight_dtype.startswith("fp8") else dtype_bytes
    if cfg.is_moe:
        experts = 3 * H * cfg.moe_intermediate_size * cfg.num_experts * w_bytes
        shared = 3 * H * cfg.moe_intermediate_size * cfg.n_shared_experts * w_bytes
        return attn * dtype_bytes + shared + H * cfg.num_experts * dtype_bytes, experts
    return attn * dtype_bytes + 3 * H * cfg.intermediate_size * dtype_bytes, 0.0


def predict(cfg: ModelConfig, m: BoxMeasurements, *, tp: int, pp: int, dp: int, batch: int,
            ctx: int, prompt: int, launches_per_layer: int = 8) -> BoxPlan:
    L = cfg.num_layers
    dense_l, expert_l = _bytes_per_layer(cfg)
    ep = tp if cfg.is_moe else 1
    H, V = cfg.hidden_size, cfg.vocab_size
    b_local = max(1, batch // dp)
    layers = math.ceil(L / pp)
    # Expert weights actually read per step: all local experts that receive a token.
    if cfg.is_moe:
        active = min(1.0, b_local * cfg.num_experts_per_tok / max(1, cfg.num_experts / ep) / 1.0)
        expert_read = expert_l / ep * max(active, 1.0 - math.exp(-b_local * cfg.num_experts_per_tok / cfg.num_experts))
    else:
        expert_read = 0.0
    w_rank = layers * (dense_l / tp + expert_read) + 2 * V * H * 2 / tp / pp
    w_store = layers * (dense_l / tp + expert_l / ep) + 2 * V * H * 2 / tp
    kv_per_token = (cfg.kv_lora_rank + cfg.qk_rope_head_dim) * 2 if cfg.mla else 2 * cfg.kv_size * 2
    kv_heads_div = 1 if cfg.mla else min(tp, cfg.num_kv_heads)
    kv_rank = b_local * ctx * layers * kv_per_token / kv_heads_div
    mem = (w_store + kv_rank * 1.1) / GB
    stream_ms = (w_rank + kv_rank) / (m.eta * m.hbm_gbs * GB) * 1e3
    launch_ms = layers * launches_per_layer * m.launch_us / 1e3
    ar_bytes = b_local * H * 2
    n_ar = 2 * layers if tp > 1 else 0
    ar_ms = n_ar * (m.ar_alpha_us + m.ar_beta_us_per_mb * ar_bytes / 1e6) / 1e3
    p2p_ms = (pp - 1) * (m.nvlink_latency_us / 1e3 + ar_bytes / (m.nvlink_gbs * GB) * 1e3)
    stage_ms = stream_ms + launch_ms + ar_ms
    flops_prefill = 2 * prompt * b_local * (cfg.parameter_count() / (tp * pp))
    ttft = flops_prefill / (m.bf16_tflops * 1e12 * 0.75) * 1e3 * pp + p2p_ms
    step = stage_ms * pp + p2p_ms  # one token traverses every stage
    # with pp micro-batches in flight the pipeline emits b_local tokens every stage time
    tok_s = dp * b_local * 1e3 / (stage_ms * max(1, pp) if b_local < pp else max(stage_ms * pp, step))
    if pp > 1 and b_local >= pp:
        tok_s = dp * b_local * 1e3 / (stage_ms * pp) * 1.0
    fits = mem <= m.gpu_memory_gb * 0.92
    unmeasured = [k for k in ("hbm_gbs", "nvlink_gbs", "ar_alpha_us", "eta", "launch_us")
                  if k not in m.measured]
    costs = score_costs(PlanCostInputs([stage_ms] * pp, [p2p_ms / max(1, pp - 1)] * (pp - 1),
                                       ttft, batch=b_local, memory_fraction=mem / m.gpu_memory_gb,
                                       unmeasured=unmeasured, replicas=dp))
    terms = {"weights_gb_read": w_rank / GB, "kv_gb_read": kv_rank / GB, "stream_ms": stream_ms,
             "launch_ms": launch_ms, "allreduce_ms": ar_ms, "pipeline_p2p_ms": p2p_ms,
             "unmeasured": unmeasured}
    return BoxPlan(tp, ep, pp, dp, step, ttft, tok_s, mem, fits, costs.score if fits else -1.0, terms)


def plan_box(cfg: ModelConfig, n_gpus: int, m: BoxMeasurements, *, batch: int, ctx: int,
             prompt: int, mode: str = "throughput") -> list[BoxPlan]:
    plans = []
    for tp in (1, 2, 4, 8):
        for pp in (1, 2, 4, 8):
            if n_gpus % (tp * pp):
                continue
            dp = n_gpus // (tp * pp)
            if cfg.num_heads % tp or (not cfg.mla and cfg.num_kv_heads % min(tp, cfg.num_kv_heads)):
                continue
            if cfg.is_moe and cfg.num_experts % tp:
                continue
            if pp > cfg.num_layers or batch < dp:
                continue
            p = predict(cfg, m, tp=tp, pp=pp, dp=dp, batch=batch, ctx=ctx, prompt=prompt)
            if mode == "speed":
                p.score = 1e3 / p.step_ms if p.fits else -1.0
            elif mode == "throughput":
                p.score = p.tokens_per_s if p.fits else -1.0
            plans.append(p)
    plans.sort(key=lambda p: -p.score)
    return plans


def explain(plans: list[BoxPlan], top: int = 5) -> str:
    lines = ["tp ep pp dp | step_ms  ttft_ms  tok/s      mem_GB fits | stream launch allreduce p2p"]
    for p in plans[:top]:
        t = p.terms
        lines.append(f"{p.tp:2d} {p.ep:2d} {p.pp:2d} {p.dp:2d} | {p.step_ms:7.3f} {p.ttft_ms:8.1f} "
                     f"{p.tokens_per_s:9.1f} {p.memory_gb_per_gpu:7.1f} {str(p.fits):5s} | "
                     f"{t['stream_ms']:.3f} {t['launch_ms']:.3f} {t['allreduce_ms']:.3f} "
                     f"{t['pipeline_p2p_ms']:.3f}")
    return "\n".join(lines)


def plan_json(p: BoxPlan) -> dict:
    return asdict(p)
