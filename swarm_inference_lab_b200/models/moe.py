"""MoE decoders (Mixtral, Qwen3-MoE; the MLP part of DeepSeek-V3/Kimi-K2) on the
sm_100a kernels.

Attention is the dense GQA block of :mod:`.dense` (tensor parallel over the
group).  The MLP is a routed expert layer:

* the router weight is replicated; every rank routes every token (the token
  activations are already replicated across the tensor-parallel group after
  the attention all-reduce, so expert dispatch needs no transfer);
* experts are sharded expert-parallel: rank r owns experts
  [r*E/ep, (r+1)*E/ep), stacked as one ``[E_local * 2I, H]`` gate/up and one
  ``[E_local * H, I]`` down weight for the grouped tcgen05 GEMM;
* assignments to remote experts are permuted into a trailing group that the
  grouped GEMM skips; the combine sums local experts' weighted outputs, and
  the group all-reduce completes the sum (with the residual added once).

Optional shared experts (DeepSeek/Kimi) and leading dense layers
(``first_k_dense``) run as dense SwiGLU blocks.

Reference: si/model/qwen3.py:1285-1325 (hybrid MoE layer, router), the
logical expert-parallel layer si/microsharding/moe.py:153-548 (ownership,
dispatch, combine) and si/execution/moe.py:433-488 (local backend).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from ..ops import gemm, moe as moe_ops
from .config import ModelConfig
from .dense import DenseLayerWeights, DenseModel, DenseWeights, TPInfo, random_tensor


@dataclass
class MoELayerWeights(DenseLayerWeights):
    router: torch.Tensor | None = None          # [E, H] bf16
    router_bias: torch.Tensor | None = None     # [E] fp32 (sigmoid routing)
    experts_gate_up: torch.Tensor | None = None  # [E_local * 2I, H]
    experts_down: torch.Tensor | None = None     # [E_local * H, I]
    shared_gate_up: torch.Tensor | None = None   # [2 * I_shared, H]
    shared_down: torch.Tensor | None = None      # [H, I_shared]
    dense: bool = False


class MoEWeights(DenseWeights):
    @classmethod
    def random(cls, cfg: ModelConfig, tp: TPInfo, device, seed: int = 0, dtype=torch.bfloat16,
               std: float = 0.02, layer_range: tuple[int, int] | None = None,
               with_embed: bool = True, with_head: bool = True) -> "MoEWeights":
        """Random N(0, std) weights (norms 1, router bias 0), generated per tensor on
        ``device`` so every expert-parallel degree sees the same model."""
        dev = torch.device(device)

        def get(name, shape):
            if name.endswith("norm.weight") or "layernorm" in name:
                return torch.ones(shape, device=dev, dtype=dtype)
            if name.endswith("e_score_correction_bias"):
                return torch.zeros(shape, device=dev, dtype=torch.float32)
            return random_tensor(shape, seed, name, dev, dtype, std)

        return cls.from_full(cfg, tp, get, device, dtype, layer_range=layer_range,
                             with_embed=with_embed, with_head=with_head)

    @classmethod
    def from_full(cls, cfg: ModelConfig, tp: TPInfo, get, device, dtype=torch.bfloat16,
                  layer_range: tuple[int, int] | None = None, with_embed: bool = True,
                  with_head: bool = True) -> "MoEWeights":
        """Shard full tensors from ``get(name, shape)`` (Hugging Face Qwen3-MoE / DeepSeek
        names; a checkpoint source maps other families onto them) for this rank: attention
        tensor parallel, experts expert parallel (rank r owns [r*E/ep, (r+1)*E/ep))."""
        dev = torch.device(device)
        H, D, E, I = cfg.hidden_size, cfg.head_dim, cfg.num_experts, cfg.moe_intermediate_size
        q0, nq = tp.heads(cfg.num_heads)
        k0, nk = tp.heads(cfg.num_kv_heads)
        ep = tp.size
        if E % ep:
            raise ValueError(f"{E} experts not divisible by expert-parallel degree {ep}")
        el = E // ep
        e0 = tp.rank * el
        lo, hi = layer_range or (0, cfg.num_layers)

        def t(name, shape):
            return get(name, shape).to(device=dev, dtype=dtype)

        layers = []
        for li in range(lo, hi):
            p = f"model.layers.{li}."
            wq = t(p + "self_attn.q_proj.weight", (cfg.num_heads * D, H))
            wk = t(p + "self_attn.k_proj.weight", (cfg.num_kv_heads * D, H))
            wv = t(p + "self_attn.v_proj.weight", (cfg.num_kv_heads * D, H))
            wqkv = torch.cat([wq[q0 * D:(q0 + nq) * D], wk[k0 * D:(k0 + nk) * D],
                              wv[k0 * D:(k0 + nk) * D]]).contiguous()
            wo = t(p + "self_attn.o_proj.weight", (H, cfg.num_heads * D))[:, q0 * D:(q0 + nq) * D].contiguous()
            L = MoELayerWeights(attn_norm=t(p + "input_layernorm.weight", (H,)).contiguous(),
                                wqkv=wqkv, wo=wo,
                                mlp_norm=t(p + "post_attention_layernorm.weight", (H,)).contiguous(),
                                w_gate_up=None, w_down=None,
                                q_norm=t(p + "self_attn.q_norm.weight", (D,)) if cfg.qk_norm else None,
                                k_norm=t(p + "self_attn.k_norm.weight", (D,)) if cfg.qk_norm else None)
            del wq, wk, wv
            if li < cfg.first_k_dense:
                i0, ni = tp.split(cfg.intermediate_size)
                g = t(p + "mlp.gate_proj.weight", (cfg.intermediate_size, H))[i0:i0 + ni]
                u = t(p + "mlp.up_proj.weight", (cfg.intermediate_size, H))[i0:i0 + ni]
                L.w_gate_up = torch.cat([g, u]).contiguous()
                L.w_down = t(p + "mlp.down_proj.weight", (H, cfg.intermediate_size))[:, i0:i0 + ni].contiguous()
                L.dense = True
            else:
                L.router = t(p + "mlp.gate.weight", (E, H)).contiguous()
                if cfg.router == "sigmoid_group":
                    L.router_bias = get(p + "mlp.gate.e_score_correction_bias", (E,)).to(
                        device=dev, dtype=torch.float32).contiguous()
                # Local experts, read one by one so any EP degree sees the same model.
                gu, dn = [], []
                for e in range(e0, e0 + el):
                    q = f"{p}mlp.experts.{e}."
                    gu.append(t(q + "gate_proj.weight", (I, H)))
                    gu.append(t(q + "up_proj.weight", (I, H)))
                    dn.append(t(q + "down_proj.weight", (H, I)))
                L.experts_gate_up = torch.cat(gu).contiguous()
                L.experts_down = torch.cat(dn).contiguous()
                del gu, dn
                if cfg.n_shared_experts:
                    Is = I * cfg.n_shared_experts
                    i0, ni = tp.split(Is)
                    g = t(p + "mlp.shared_experts.gate_proj.weight", (Is, H))[i0:i0 + ni]
                    u = t(p + "mlp.shared_experts.up_proj.weight", (Is, H))[i0:i0 + ni]
                    L.shared_gate_up = torch.cat([g, u]).contiguous()
                    L.shared_down = t(p + "mlp.shared_experts.down_proj.weight", (H, Is))[:, i0:i0 + ni].contiguous()
            layers.append(L)
        embed = t("model.embed_tokens.weight", (cfg.vocab_size, H)).contiguous() if with_embed else None
        final_norm = lm_head = None
        v0 = 0
        if with_head:
            final_norm = t("model.norm.weight", (H,)).contiguous()
            v0, nv = tp.split(cfg.vocab_size)
            name = "model.embed_tokens.weight" if cfg.tie_word_embeddings else "lm_head.weight"
            lm_head = t(name, (cfg.vocab_size, H))[v0:v0 + nv].contiguous()
        w = cls(cfg, tp, embed, layers, final_norm, lm_head, v0)
        w.expert_start = e0
        w.experts_local = el
        return w


class MoEModel(DenseModel):
    """Dense attention + routed-expert MLP; see module docstring."""

    def __init__(self, weights: MoEWeights, device, comm=None, max_positions: int | None = None):
        super().__init__(weights, device, comm=comm, max_positions=max_positions)
        self.e0 = weights.expert_start
        self.el = weights.experts_local
        cfg = self.cfg
        self.mode = moe_ops.MODE_SIGMOID_GROUP if cfg.router == "sigmoid_group" else moe_ops.MODE_SOFTMAX
        self.route_scale = cfg.routed_scaling_factor if cfg.router == "sigmoid_group" else 1.0

    def mlp(self, li: int, L, x: torch.Tensor, h: torch.Tensor):
        if getattr(L, "dense", True) and L.router is None:
            return super().mlp(li, L, x, h)
        cfg = self.cfg
        T = x.shape[0]
        k = cfg.num_experts_per_tok
        logits = gemm.linear(x, L.router, fp32_out=True)
        ids, w = moe_ops.route(logits, k, mode=self.mode, renorm=cfg.norm_topk_prob,
                               bias=L.router_bias, n_group=cfg.n_group, topk_group=cfg.topk_group,
                               scale=self.route_scale)
        if self.tp.size > 1:
            # Global expert id -> local group; remote experts go to the trailing group.
            local = ids - self.e0
            ids = torch.where((local >= 0) & (local < self.el), local,
                              torch.full_like(local, self.el))
        offsets, rows, _ = moe_ops.permute(ids, self.el + 1)
        xp = moe_ops.gather(x, rows, k)
        hint = max(1, (T * k + cfg.num_experts - 1) // cfg.num_experts)
        act = moe_ops.grouped_linear(xp, L.experts_gate_up, offsets, self.el, swiglu=True,
                                     rows_hint=hint)
        y = moe_ops.grouped_linear(act, L.experts_down, offsets, self.el, rows_hint=hint)
        shared = None
        if L.shared_gate_up is not None:
            sa = gemm.linear(x, L.shared_gate_up, swiglu=True)
            shared = gemm.linear(sa, L.shared_down)
        limit = offsets[self.el:self.el + 1]
        if self.tp.size == 1:
            moe_ops.combine(y, rows, w, k, residual=h, shared=shared, out=h, row_limit=limit)
            return None
        buf = getattr(self.comm, "partial_buffer", None)
        dst = buf(T, x.shape[1]) if buf is not None and h.is_contiguous() else None
        if dst is not None:
            # Expert parallelism over NVLink: the combine of this rank's experts lands in its
            # symmetric partial buffer and the low-latency all-reduce adds every rank's
            # partial to the residual stream in rank order.
            moe_ops.combine(y, rows, w, k, shared=shared, row_limit=limit, out=dst)
            self.comm.allreduce_partial_residual(h)
            return None
        part = moe_ops.combine(y, rows, w, k, shared=shared, row_limit=limit)
        return self._reduce(part)
