"""Plain-PyTorch decoder used as the numerical oracle and as the CPU stage backend.

Runs any device / dtype (fp32 on CPU for the loopback pipeline, fp32 on the
GPU as the oracle of the sm_100a kernels).  Weights come from the same
``get(name, shape)`` source as the GPU model, in Hugging Face tensor names,
so a seed or a safetensors checkpoint yields identical numbers on both.

Supports a contiguous per-sequence KV cache for incremental decode over a
layer interval, which is what a pipeline stage owner needs: stage 0 embeds,
the last stage applies the final norm and LM head (si/model/qwen3.py:1585-1703).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from ..ops.rope import rope_cos_sin_table
from .config import ModelConfig


def _rms(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    var = xf.pow(2).mean(-1, keepdim=True)
    return (w.float() * (xf * torch.rsqrt(var + eps)).to(x.dtype).float()).to(x.dtype)


def _rope(x: torch.Tensor, cs: torch.Tensor) -> torch.Tensor:
    # x: [T, H, D]; cs: [T, D] (cos | sin halves)
    d = x.shape[-1]
    cos, sin = cs[:, None, : d // 2], cs[:, None, d // 2:]
    xf = x.float()
    x1, x2 = xf[..., : d // 2], xf[..., d // 2:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1).to(x.dtype)


@dataclass
class RefCache:
    k: list = field(default_factory=list)  # per local layer [T, Hkv, D]
    v: list = field(default_factory=list)

    @property
    def length(self) -> int:
        return 0 if not self.k else self.k[0].shape[0]

    def truncate(self, n: int) -> None:
        self.k = [t[:n] for t in self.k]
        self.v = [t[:n] for t in self.v]

    def clone(self) -> "RefCache":
        return RefCache([t.clone() for t in self.k], [t.clone() for t in self.v])


class ReferenceDecoder:
    """Dense GQA decoder (llama / mistral / qwen3) over layers [lo, hi)."""

    def __init__(self, cfg: ModelConfig, get, *, device="cpu", dtype=torch.float32,
                 layer_range: tuple[int, int] | None = None, with_embed: bool | None = None,
                 with_head: bool | None = None, max_positions: int | None = None):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype
        lo, hi = layer_range or (0, cfg.num_layers)
        self.lo, self.hi = lo, hi
        self.with_embed = (lo == 0) if with_embed is None else with_embed
        self.with_head = (hi == cfg.num_layers) if with_head is None else with_head

        def t(name, shape):
            return get(name, shape).to(device=self.device, dtype=dtype)

        H, D = cfg.hidden_size, cfg.head_dim
        self.layers = []
        for li in range(lo, hi):
            p = f"model.layers.{li}."
            L = {
                "index": li,
                "ln1": t(p + "input_layernorm.weight", (H,)),
                "wq": t(p + "self_attn.q_proj.weight", (cfg.num_heads * D, H)),
                "wk": t(p + "self_attn.k_proj.weight", (cfg.num_kv_heads * D, H)),
                "wv": t(p + "self_attn.v_proj.weight", (cfg.num_kv_heads * D, H)),
                "wo": t(p + "self_attn.o_proj.weight", (H, cfg.num_heads * D)),
                "ln2": t(p + "post_attention_layernorm.weight", (H,)),
            }
            if cfg.is_moe and li >= cfg.first_k_dense:
                E, I = cfg.num_experts, cfg.moe_intermediate_size
                L["router"] = t(p + "mlp.gate.weight", (E, H))
                L["experts"] = [(t(f"{p}mlp.experts.{e}.gate_proj.weight", (I, H)),
                                 t(f"{p}mlp.experts.{e}.up_proj.weight", (I, H)),
                                 t(f"{p}mlp.experts.{e}.down_proj.weight", (H, I))) for e in range(E)]
                if cfg.n_shared_experts:
                    Is = I * cfg.n_shared_experts
                    L["shared"] = (t(p + "mlp.shared_experts.gate_proj.weight", (Is, H)),
                                   t(p + "mlp.shared_experts.up_proj.weight", (Is, H)),
                                   t(p + "mlp.shared_experts.down_proj.weight", (H, Is)))
            else:
                L["wg"] = t(p + "mlp.gate_proj.weight", (cfg.intermediate_size, H))
                L["wu"] = t(p + "mlp.up_proj.weight", (cfg.intermediate_size, H))
                L["wd"] = t(p + "mlp.down_proj.weight", (H, cfg.intermediate_size))
            if cfg.qk_norm:
                L["qn"] = t(p + "self_attn.q_norm.weight", (D,))
                L["kn"] = t(p + "self_attn.k_norm.weight", (D,))
            self.layers.append(L)
        self.embed = t("model.embed_tokens.weight", (cfg.vocab_size, H)) if self.with_embed else None
        if self.with_head:
            self.norm = t("model.norm.weight", (H,))
            name = "model.embed_tokens.weight" if cfg.tie_word_embeddings else "lm_head.weight"
            self.lm_head = t(name, (cfg.vocab_size, H))
        mp = max_positions or cfg.max_position_embeddings
        self.cos_sin = rope_cos_sin_table(mp, D, cfg.rope_theta, cfg.rope_scaling).to(self.device)

    # Where the routed experts run (``runtime/moe_backends.py``); None: the experts held here.
    moe_backend = None

    def _moe(self, L, m: torch.Tensor) -> torch.Tensor:
        from ..ops.moe import MODE_SIGMOID_GROUP, MODE_SOFTMAX, route_reference
        cfg = self.cfg
        sig = cfg.router == "sigmoid_group"
        ids, w = route_reference(m.float() @ L["router"].float().T, cfg.num_experts_per_tok,
                                 mode=MODE_SIGMOID_GROUP if sig else MODE_SOFTMAX,
                                 renorm=cfg.norm_topk_prob, n_group=cfg.n_group,
                                 topk_group=cfg.topk_group,
                                 scale=cfg.routed_scaling_factor if sig else 1.0)
        if self.moe_backend is not None:
            out = self.moe_backend.experts(L["index"], m.float().cpu(), ids.cpu(), w.float().cpu())
            out = out.to(m.device)
            if "shared" in L:
                g, u, d = L["shared"]
                out += ((torch.nn.functional.silu(m @ g.T) * (m @ u.T)) @ d.T).float()
            return out.to(m.dtype)
        out = torch.zeros_like(m, dtype=torch.float32)
        for e in torch.unique(ids).tolist():
            sel = (ids == e)
            tok = sel.any(-1).nonzero().squeeze(-1)
            we = (w * sel).sum(-1)[tok]
            g, u, d = L["experts"][e]
            xe = m[tok]
            ye = (torch.nn.functional.silu(xe @ g.T) * (xe @ u.T)) @ d.T
            out.index_add_(0, tok, we[:, None].float() * ye.float())
        if "shared" in L:
            g, u, d = L["shared"]
            out += ((torch.nn.functional.silu(m @ g.T) * (m @ u.T)) @ d.T).float()
        return out.to(m.dtype)

    def new_cache(self) -> RefCache:
        return RefCache()

    @torch.no_grad()
    def forward(self, x: torch.Tensor, cache: RefCache | None = None) -> torch.Tensor:
        """x: token ids [T] (first stage) or hidden states [T, H].  Appends to ``cache``.
        Returns hidden states [T, H] (inner stage) or logits [T, V] (last stage)."""
        cfg = self.cfg
        if self.with_embed:
            h = self.embed[x.to(self.device).long()]
        else:
            h = x.to(device=self.device, dtype=self.dtype)
        T = h.shape[0]
        start = cache.length if cache is not None else 0
        pos = torch.arange(start, start + T, device=self.device)
        cs = self.cos_sin[pos]
        D, nq, nkv = cfg.head_dim, cfg.num_heads, cfg.num_kv_heads
        g = nq // nkv
        scale = 1.0 / math.sqrt(D)
        eps = cfg.rms_norm_eps
        for i, L in enumerate(self.layers):
            a = _rms(h, L["ln1"], eps)
            q = (a @ L["wq"].T).view(T, nq, D)
            k = (a @ L["wk"].T).view(T, nkv, D)
            v = (a @ L["wv"].T).view(T, nkv, D)
            if cfg.qk_norm:
                q = _rms(q, L["qn"], eps)
                k = _rms(k, L["kn"], eps)
            q, k = _rope(q, cs), _rope(k, cs)
            if cache is not None:
                if len(cache.k) <= i:
                    cache.k.append(k)
                    cache.v.append(v)
                else:
                    cache.k[i] = torch.cat([cache.k[i], k])
                    cache.v[i] = torch.cat([cache.v[i], v])
                kk, vv = cache.k[i], cache.v[i]
            else:
                kk, vv = k, v
            Tk = kk.shape[0]
            kf = kk.float().repeat_interleave(g, dim=1)
            vf = vv.float().repeat_interleave(g, dim=1)
            s = torch.einsum("qhd,khd->hqk", q.float(), kf) * scale
            qpos = pos[:, None]
            kpos = torch.arange(Tk, device=self.device)[None, :]
            s = s.masked_fill((kpos > qpos)[None], float("-inf"))
            o = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), vf).to(self.dtype)
            h = h + o.reshape(T, nq * D) @ L["wo"].T
            m = _rms(h, L["ln2"], eps)
            if "router" in L:
                h = h + self._moe(L, m)
            else:
                act = torch.nn.functional.silu(m @ L["wg"].T) * (m @ L["wu"].T)
                h = h + act @ L["wd"].T
        if not self.with_head:
            return h
        return (_rms(h, self.norm, eps).float() @ self.lm_head.float().T)

    @torch.no_grad()
    def greedy_generate(self, prompt: list[int], max_new_tokens: int) -> tuple[list[int], list[torch.Tensor]]:
        """Whole-model greedy decode (needs embed and head).  Returns tokens and per-step logits."""
        cache = self.new_cache()
        logits = self.forward(torch.tensor(prompt), cache)[-1]
        out, all_logits = [], [logits]
        for _ in range(max_new_tokens):
            tok = int(torch.argmax(logits))
            out.append(tok)
            if len(out) == max_new_tokens:
                break
            logits = self.forward(torch.tensor([tok]), cache)[-1]
            all_logits.append(logits)
        return out, all_logits


def random_source(seed: int, std: float = 0.02, device="cpu"):
    """``get(name, shape)`` producing the deterministic random weights used everywhere."""
    from .dense import random_tensor

    def get(name, shape):
        if name.endswith("norm.weight") or "layernorm" in name:
            return torch.ones(shape, dtype=torch.float32, device=device)
        return random_tensor(shape, seed, name, torch.device(device), torch.float32, std)

    return get
