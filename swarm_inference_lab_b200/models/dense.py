"""Dense GQA decoder (Llama / Mistral / Qwen3) on the sm_100a kernels.

Weights live on one GPU per tensor-parallel rank, in the layout the kernels
want: a fused ``[q; k; v]`` projection (column parallel), ``wo`` (row
parallel), a fused ``[gate; up]`` projection for the SwiGLU epilogue (column
parallel), ``w_down`` (row parallel) and a vocabulary-parallel LM head.  The
embedding table is replicated (a gather needs no communication).

Per layer the forward pass is 5 launches at TP=1 (norm, QKV GEMM,
RoPE+KV-write, attention, O GEMM with fused residual add) + 3 for the MLP
(norm, gate/up GEMM with fused SwiGLU, down GEMM with fused residual add).
With TP > 1 the row-parallel GEMMs hand their partial sums to the group's
all-reduce (fused GEMM+all-reduce kernel, or NCCL as the baseline) and the
residual add moves into the following RMSNorm.

Reference: the per-layer structure of HF ``Qwen3DecoderLayer`` used by
si/model/qwen3.py:517-546 and the Megatron split of the logical TP model in
si/microsharding/dense.py:222-412, 575-760 (column-parallel q/k/v and
gate/up, row-parallel o/down, vocabulary-parallel head with lowest-id
distributed argmax, :763-838).
"""
from __future__ import annotations

import hashlib
import math
from dataclasses import dataclass

import torch

from ..ops import attention as attn_ops
from ..ops import gemm, norm, rope, sampling
from .config import ModelConfig


def tensor_seed(seed: int, name: str) -> int:
    """Deterministic per-tensor seed, identical on every rank and TP degree."""
    h = hashlib.sha256(f"{seed}:{name}".encode()).digest()
    return int.from_bytes(h[:8], "little") & ((1 << 63) - 1)


def random_tensor(shape, seed: int, name: str, device, dtype, std: float = 0.02) -> torch.Tensor:
    gen = torch.Generator(device=device)
    gen.manual_seed(tensor_seed(seed, name))
    t = torch.empty(shape, device=device, dtype=torch.float32)
    t.normal_(0.0, std, generator=gen)
    return t.to(dtype)


@dataclass
class TPInfo:
    rank: int = 0
    size: int = 1

    def heads(self, n: int) -> tuple[int, int]:
        """Local [start, count) of `n` heads; heads are replicated when n < size."""
        if n >= self.size:
            assert n % self.size == 0, f"{n} heads not divisible by TP {self.size}"
            per = n // self.size
            return self.rank * per, per
        return self.rank * n // self.size, 1

    def split(self, n: int) -> tuple[int, int]:
        assert n % self.size == 0, f"{n} not divisible by TP {self.size}"
        per = n // self.size
        return self.rank * per, per


@dataclass
class DenseLayerWeights:
    attn_norm: torch.Tensor
    wqkv: torch.Tensor
    wo: torch.Tensor
    mlp_norm: torch.Tensor
    w_gate_up: torch.Tensor
    w_down: torch.Tensor
    q_norm: torch.Tensor | None = None
    k_norm: torch.Tensor | None = None


class DenseWeights:
    """Rank-local weights of a dense decoder."""

    def __init__(self, cfg: ModelConfig, tp: TPInfo, embed, layers, final_norm, lm_head,
                 vocab_start: int):
        self.cfg = cfg
        self.tp = tp
        self.embed = embed
        self.layers: list[DenseLayerWeights] = layers
        self.final_norm = final_norm
        self.lm_head = lm_head
        self.vocab_start = vocab_start

    @classmethod
    def from_full(cls, cfg: ModelConfig, tp: TPInfo, get, device, dtype=torch.bfloat16,
                  layer_range: tuple[int, int] | None = None, with_embed: bool = True,
                  with_head: bool = True) -> "DenseWeights":
        """Shard full tensors produced by ``get(name, shape)`` (HF names) for this rank."""
        H, D = cfg.hidden_size, cfg.head_dim
        q0, nq = tp.heads(cfg.num_heads)
        k0, nk = tp.heads(cfg.num_kv_heads)
        i0, ni = tp.split(cfg.intermediate_size)
        lo, hi = layer_range or (0, cfg.num_layers)

        def dev(t):
            return t.to(device=device, dtype=dtype).contiguous()

        layers = []
        for li in range(lo, hi):
            p = f"model.layers.{li}."
            wq = get(p + "self_attn.q_proj.weight", (cfg.num_heads * D, H))
            wk = get(p + "self_attn.k_proj.weight", (cfg.num_kv_heads * D, H))
            wv = get(p + "self_attn.v_proj.weight", (cfg.num_kv_heads * D, H))
            wqkv = torch.cat([wq[q0 * D:(q0 + nq) * D], wk[k0 * D:(k0 + nk) * D],
                              wv[k0 * D:(k0 + nk) * D]], dim=0)
            wo = get(p + "self_attn.o_proj.weight", (H, cfg.num_heads * D))[:, q0 * D:(q0 + nq) * D]
            gate = get(p + "mlp.gate_proj.weight", (cfg.intermediate_size, H))[i0:i0 + ni]
            up = get(p + "mlp.up_proj.weight", (cfg.intermediate_size, H))[i0:i0 + ni]
            down = get(p + "mlp.down_proj.weight", (H, cfg.intermediate_size))[:, i0:i0 + ni]
            layers.append(DenseLayerWeights(
                attn_norm=dev(get(p + "input_layernorm.weight", (H,))),
                wqkv=dev(wqkv), wo=dev(wo),
                mlp_norm=dev(get(p + "post_attention_layernorm.weight", (H,))),
                w_gate_up=dev(torch.cat([gate, up], dim=0)), w_down=dev(down),
                q_norm=dev(get(p + "self_attn.q_norm.weight", (D,))) if cfg.qk_norm else None,
                k_norm=dev(get(p + "self_attn.k_norm.weight", (D,))) if cfg.qk_norm else None,
            ))
            del wq, wk, wv, wqkv, wo, gate, up, down
        embed = dev(get("model.embed_tokens.weight", (cfg.vocab_size, H))) if with_embed else None
        final_norm = lm_head = None
        v0 = 0
        if with_head:
            final_norm = dev(get("model.norm.weight", (H,)))
            v0, nv = tp.split(cfg.vocab_size)
            name = "model.embed_tokens.weight" if cfg.tie_word_embeddings else "lm_head.weight"
            lm_head = dev(get(name, (cfg.vocab_size, H))[v0:v0 + nv])
        return cls(cfg, tp, embed, layers, final_norm, lm_head, v0)

    @classmethod
    def random(cls, cfg: ModelConfig, tp: TPInfo, device, seed: int = 0, dtype=torch.bfloat16,
               std: float = 0.02, **kw) -> "DenseWeights":
        """Random N(0, std) weights (norm weights = 1), generated per tensor on ``device``
        from ``seed`` so every TP degree and rank sees the same full model."""
        gen_device = torch.device(device)

        def get(name, shape):
            if name.endswith("norm.weight") or "layernorm" in name:
                return torch.ones(shape, device=gen_device, dtype=torch.float32)
            return random_tensor(shape, seed, name, gen_device, torch.float32, std)

        return cls.from_full(cfg, tp, get, device, dtype, **kw)

    def nbytes(self) -> int:
        """Bytes of every weight tensor held, including (codes, scales) pairs of quantized
        weights; flags and other non-tensor layer attributes are skipped."""
        def size(t) -> int:
            if isinstance(t, torch.Tensor):
                return t.numel() * t.element_size()
            if isinstance(t, (tuple, list)):
                return sum(size(u) for u in t)
            return 0
        n = sum(size(t) for t in [self.embed, self.final_norm, self.lm_head])
        for L in self.layers:
            n += sum(size(t) for t in vars(L).values())
        return n


@dataclass
class ForwardBatch:
    """Device-side metadata of one forward pass (prefill or decode)."""

    ids: torch.Tensor          # [T] int64
    positions: torch.Tensor    # [T] int32
    slots: torch.Tensor        # [T] int32 (page * 64 + offset; -1 skips the KV write)
    seq_lens: torch.Tensor     # [B] int32 (context length after this step)
    block_table: torch.Tensor  # [B, max_pages] int32
    last_idx: torch.Tensor     # [B] int64 rows whose logits are needed
    is_decode: bool
    cu_q: torch.Tensor | None = None   # [B+1] int32 (prefill)
    max_q_len: int = 1
    decode_splits: int = 1


class DenseModel:
    """Forward pass of a dense decoder over a paged KV cache (one rank)."""

    def __init__(self, weights: DenseWeights, device, comm=None, max_positions: int | None = None,
                 is_first: bool = True, is_last: bool = True):
        self.w = weights
        self.cfg = weights.cfg
        self.tp = weights.tp
        self.device = torch.device(device)
        self.comm = comm
        self.is_first = is_first
        self.is_last = is_last
        cfg = self.cfg
        if cfg.head_dim != 128:
            raise ValueError("the sm_100a attention kernels need head_dim == 128")
        self.num_q_local = self.tp.heads(cfg.num_heads)[1]
        self.num_kv_local = self.tp.heads(cfg.num_kv_heads)[1]
        mp = max_positions or cfg.max_position_embeddings
        self.cos_sin = rope.rope_cos_sin_table(mp, cfg.head_dim, cfg.rope_theta, cfg.rope_scaling,
                                               device=self.device)
        self.scale = 1.0 / math.sqrt(cfg.head_dim)

    @property
    def num_layers(self) -> int:
        return len(self.w.layers)

    def _reduce(self, x: torch.Tensor) -> torch.Tensor:
        if self.tp.size > 1:
            self.comm.all_reduce(x)
        return x

    def _row_parallel(self, x: torch.Tensor, w: torch.Tensor, h: torch.Tensor):
        """x @ w.T reduced over the TP group.  Returns the partial to add into h
        (None when the add was fused into the GEMM epilogue at TP=1)."""
        if self.tp.size == 1:
            gemm.linear(x, w, out=h, residual=h)
            return None
        fused = getattr(self.comm, "fused_gemm_allreduce_residual", None)
        if fused is not None:
            return fused(x, w, h)  # h += allreduce(x @ w.T) in one kernel
        out = gemm.linear(x, w)
        return self._reduce(out)

    def mlp(self, li: int, L, x: torch.Tensor, h: torch.Tensor):
        """SwiGLU MLP on the normalised input ``x``; adds into ``h`` (returns None) or
        returns the partial sum still to be added by the next norm."""
        act = gemm.linear(x, L.w_gate_up, swiglu=True)
        return self._row_parallel(act, L.w_down, h)

    sequence_parallel = False  # prefill: shard the residual stream over tokens between TP blocks

    def _forward_hidden_sp(self, fb: ForwardBatch, kv) -> torch.Tensor:
        """Sequence-parallel prefill: between tensor-parallel blocks the residual stream is
        sharded over tokens (rank r holds rows [r*T/tp, (r+1)*T/tp)), so RMSNorm runs on a
        1/tp slice; each block all-gathers its normalised input and reduce-scatters its
        row-parallel output (the same bytes as one all-reduce).  Reference semantics:
        si/microsharding/sequence_parallel.py:20-81 (prefill only)."""
        cfg = self.cfg
        tp, r = self.tp.size, self.tp.rank
        eps = cfg.rms_norm_eps
        nq, nkv, D = self.num_q_local, self.num_kv_local, cfg.head_dim
        full = sampling.embedding(fb.ids, self.w.embed)
        T, H = full.shape
        Ts = T // tp
        h = full[r * Ts:(r + 1) * Ts].contiguous()
        xl = torch.empty_like(h)
        pending = None
        for li, L in enumerate(self.w.layers):
            if pending is None:
                norm.rmsnorm(h, L.attn_norm, eps, out=xl)
            else:
                norm.rmsnorm(pending, L.attn_norm, eps, out=xl, residual=h)
            x = self.comm.all_gather(xl).view(T, H)
            qkv = gemm.linear(x, L.wqkv)
            k_cache, v_cache = kv.layer(li)
            rope.rope_kv_write(qkv, fb.positions, fb.slots, self.cos_sin, k_cache, v_cache, nq, nkv,
                               L.q_norm, L.k_norm, eps)
            q = qkv.as_strided((T, nq, D), (qkv.stride(0), D, 1))
            a = attn_ops.paged_prefill(q, k_cache, v_cache, fb.block_table, fb.seq_lens, fb.cu_q,
                                       fb.max_q_len, scale=self.scale)
            pending = self.comm.reduce_scatter(gemm.linear(a, L.wo))
            norm.rmsnorm(pending, L.mlp_norm, eps, out=xl, residual=h)
            x = self.comm.all_gather(xl).view(T, H)
            act = gemm.linear(x, L.w_gate_up, swiglu=True)
            pending = self.comm.reduce_scatter(gemm.linear(act, L.w_down))
        h.add_(pending)
        return self.comm.all_gather(h).view(T, H)

    def forward_hidden(self, fb: ForwardBatch, kv, h: torch.Tensor | None = None) -> torch.Tensor:
        """Run the local layers; returns the residual stream ``h`` [T, H] (bf16)."""
        cfg = self.cfg
        if (h is None and self.sequence_parallel and not fb.is_decode and self.tp.size > 1
                and fb.ids.shape[0] % self.tp.size == 0 and type(self).mlp is DenseModel.mlp
                and self.w.layers):
            return self._forward_hidden_sp(fb, kv)
        if h is None:
            h = sampling.embedding(fb.ids, self.w.embed)
        T = h.shape[0]
        eps = cfg.rms_norm_eps
        nq, nkv, D = self.num_q_local, self.num_kv_local, cfg.head_dim
        pending = None
        x = torch.empty_like(h)
        # With a communicator that fuses the all-reduce with the following RMSNorm, every
        # row-parallel projection also produces the next block's normalised input.
        ar_norm = (getattr(self.comm, "fused_gemm_allreduce_residual_norm", None)
                   if self.tp.size > 1 and type(self).mlp is DenseModel.mlp else None)
        x_ready = False
        layers = self.w.layers
        for li, L in enumerate(layers):
            if x_ready:
                x_ready = False
            elif pending is None:
                norm.rmsnorm(h, L.attn_norm, eps, out=x)
            else:
                norm.rmsnorm(pending, L.attn_norm, eps, out=x, residual=h)
            qkv = gemm.linear(x, L.wqkv)
            k_cache, v_cache = kv.layer(li)
            rope.rope_kv_write(qkv, fb.positions, fb.slots, self.cos_sin, k_cache, v_cache, nq, nkv,
                               L.q_norm, L.k_norm, eps)
            q = qkv.as_strided((T, nq, D), (qkv.stride(0), D, 1))
            if fb.is_decode:
                a = attn_ops.paged_decode(q, k_cache, v_cache, fb.block_table, fb.seq_lens,
                                          num_splits=fb.decode_splits, scale=self.scale)
            else:
                a = attn_ops.paged_prefill(q, k_cache, v_cache, fb.block_table, fb.seq_lens,
                                           fb.cu_q, fb.max_q_len, scale=self.scale)
            if ar_norm is not None:
                ar_norm(a, L.wo, h, L.mlp_norm, eps, x)
                act = gemm.linear(x, L.w_gate_up, swiglu=True)
                if li + 1 < len(layers):
                    ar_norm(act, L.w_down, h, layers[li + 1].attn_norm, eps, x)
                    x_ready = True
                else:
                    self.comm.fused_gemm_allreduce_residual(act, L.w_down, h)
                pending = None
                continue
            pending = self._row_parallel(a, L.wo, h)
            if pending is None:
                norm.rmsnorm(h, L.mlp_norm, eps, out=x)
            else:
                norm.rmsnorm(pending, L.mlp_norm, eps, out=x, residual=h)
            pending = self.mlp(li, L, x, h)
        if pending is not None:
            h.add_(pending)
        return h

    def logits(self, h: torch.Tensor, fb: ForwardBatch) -> torch.Tensor:
        """fp32 logits of this rank's vocabulary shard for rows ``fb.last_idx``."""
        hl = h.index_select(0, fb.last_idx) if h.shape[0] != fb.last_idx.shape[0] else h
        x = norm.rmsnorm(hl, self.w.final_norm, self.cfg.rms_norm_eps)
        return gemm.linear(x, self.w.lm_head, fp32_out=True)

    def greedy(self, logits: torch.Tensor) -> torch.Tensor:
        """Greedy token per row; under TP a distributed argmax with lowest-id ties."""
        idx = sampling.argmax(logits)
        if self.tp.size == 1:
            return idx
        exchange = getattr(self.comm, "argmax_exchange", None)
        if exchange is not None:
            out = exchange(logits, idx, self.w.vocab_start)
            if out is not None:
                return out
        val = logits.gather(1, idx[:, None]).squeeze(1)
        gid = (idx + self.w.vocab_start).to(torch.float32)
        pair = torch.stack([val, gid], dim=1)  # [B, 2] (ids < 2^24 are exact in fp32)
        allp = self.comm.all_gather(pair)       # [tp, B, 2]
        vals, ids = allp[..., 0], allp[..., 1]
        best = vals.max(dim=0).values
        cand = torch.where(vals == best[None], ids, torch.full_like(ids, float("inf")))
        return cand.min(dim=0).values.to(torch.int64)

    def forward(self, fb: ForwardBatch, kv) -> torch.Tensor:
        h = self.forward_hidden(fb, kv)
        return self.greedy(self.logits(h, fb))
