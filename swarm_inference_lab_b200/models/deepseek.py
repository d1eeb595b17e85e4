"""DeepSeek-V3 / Kimi-K2 decoder: MLA attention over a latent paged cache, block-scaled
fp8 (e4m3, 128x128 weight / 1x128 activation scales) projections, sigmoid-routed
experts with a correction bias and group-limited top-k, one shared expert, leading
dense layers.

Parallel layout on one box (``ep`` = ranks of the group):

* attention is data parallel: each rank owns its own sequences, their latent KV
  pages and a replica of the attention / dense weights (MLA's cache is shared by
  all heads, so head sharding would replicate the cache instead);
* routed experts are sharded contiguously over the ranks (expert parallel).
  Decode with a fused communicator (``parallel/fused_ep.py``): each rank routes
  its own tokens and pushes them in e4m3 to every expert owner over peer
  memory; the owners' grouped down projection writes the weighted results
  straight back into the tokens' owners (combine fused into the epilogue).
  Otherwise (prefill, NCCL baseline): all-gather of the normalised tokens,
  replicated routing, local experts, reduce-scatter of the weighted combine;
* the shared expert and the dense layers run on the local tokens.

Forward of one layer (T local tokens, Hh heads):

    x = rmsnorm(h)
    [q_a | kv_a] = fp8(x) @ W_qkv_a            (one GEMM, 1536 + 576 rows, padded to 128)
    q = fp8(rmsnorm(q_a)) @ W_q_b              -> per head nope(128) | rope(64)
    cache[slot] = rmsnorm(c_kv) | rope(k_pe)   (mla.kv_write)
    q_lat[h] = W_UK[h]^T q_nope[h]             (grouped GEMM over heads)
    o_lat = MLA(q_lat, q_pe, cache)            (absorbed paged attention)
    o[h] = W_UV[h] o_lat[h]                    (grouped GEMM over heads)
    h += fp8(o) @ W_o                          (residual fused in the epilogue)
    h += MoE(rmsnorm(h))  or dense SwiGLU

The reference profiles these families only (si/model/architecture_adapters.py:735-976,
si/backends/colibri/sparse_moe.py:60-218 for the router and fp8 block-scale semantics).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from ..ops import fp8, gemm, mla, norm, rope, sampling
from ..ops import moe as moe_ops
from .config import ModelConfig
from .dense import ForwardBatch, TPInfo, random_tensor, tensor_seed

FP8 = tuple  # (e4m3 codes uint8 [N, K], fp32 scales [N/128, K/128])


def _pad128(n: int) -> int:
    return (n + 127) // 128 * 128


def random_fp8(shape, seed: int, name: str, device, std: float = 0.02, chunk_rows: int = 4096) -> FP8:
    """Random N(0, std) weight quantised to e4m3 with 128x128 block scales, built in
    row chunks so large tensors never exist in fp32 at full size."""
    N, K = shape
    q = torch.empty((N, K), dtype=torch.uint8, device=device)
    s = torch.empty((N // 128, K // 128), dtype=torch.float32, device=device)
    gen = torch.Generator(device=device)
    gen.manual_seed(tensor_seed(seed, name))
    for r0 in range(0, N, chunk_rows):
        r1 = min(N, r0 + chunk_rows)
        w = torch.empty((r1 - r0, K), dtype=torch.float32, device=device)
        w.normal_(0.0, std, generator=gen)
        qq, ss = fp8.quantize_weight(w)
        q[r0:r1].copy_(qq)
        s[r0 // 128:r1 // 128].copy_(ss)
    return q, s


def cat_fp8(parts: list[FP8]) -> FP8:
    return torch.cat([p[0] for p in parts]).contiguous(), torch.cat([p[1] for p in parts]).contiguous()


def pad_rows_fp8(w: FP8, rows: int) -> FP8:
    q, s = w
    if q.shape[0] == rows:
        return w
    qp = torch.zeros((rows, q.shape[1]), dtype=q.dtype, device=q.device)
    qp[: q.shape[0]] = q
    sp = torch.ones((rows // 128, s.shape[1]), dtype=s.dtype, device=s.device)
    sp[: s.shape[0]] = s
    return qp, sp


@dataclass
class MLALayerWeights:
    attn_norm: torch.Tensor
    w_qkv_a: FP8               # [pad128(q_lora + kv_lora + rope), H]
    q_a_norm: torch.Tensor     # [q_lora] bf16
    w_q_b: FP8                 # [Hh * (nope + rope), q_lora]
    kv_a_norm: torch.Tensor    # [kv_lora] fp32
    w_uk: torch.Tensor         # [Hh * kv_lora, nope] bf16 (W_UK[h]^T stacked)
    w_uv: torch.Tensor         # [Hh * v, kv_lora] bf16
    w_o: FP8                   # [H, Hh * v]
    mlp_norm: torch.Tensor
    dense: bool = True
    w_gate_up: FP8 | None = None
    w_down: FP8 | None = None
    router: torch.Tensor | None = None       # [E, H] bf16
    router_bias: torch.Tensor | None = None  # [E] fp32
    experts_gate_up: FP8 | None = None       # [El * 2I, H]
    experts_down: FP8 | None = None          # [El * H, I]
    shared_gate_up: FP8 | None = None
    shared_down: FP8 | None = None


@dataclass
class MLAWeights:
    cfg: ModelConfig
    ep: TPInfo
    embed: torch.Tensor
    layers: list[MLALayerWeights]
    final_norm: torch.Tensor
    lm_head: torch.Tensor
    expert_start: int = 0
    experts_local: int = 0

    @classmethod
    def random(cls, cfg: ModelConfig, ep: TPInfo, device, seed: int = 0,
               num_layers: int | None = None) -> "MLAWeights":
        """Random N(0, 0.02) weights (norms 1; router bias N(0, 0.01)); projections are
        quantised to e4m3 with 128x128 block scales."""
        dev = torch.device(device)

        def get(name, shape, dtype=torch.bfloat16):
            if name.endswith("norm.weight") or "layernorm" in name:
                return torch.ones(shape, dtype=dtype, device=dev)
            std = 0.01 if name.endswith("e_score_correction_bias") else 0.02
            return random_tensor(shape, seed, name, dev, dtype, std)

        def fp8w(name, shape):
            # Rows padded to a whole 128-row scale block (the padding rows are never read).
            return random_fp8((_pad128(shape[0]), shape[1]), seed, name, dev)

        return cls.from_source(cfg, ep, get, fp8w, dev, num_layers=num_layers)

    @classmethod
    def from_source(cls, cfg: ModelConfig, ep: TPInfo, get, fp8w, device,
                    num_layers: int | None = None) -> "MLAWeights":
        """Builds this rank's weights from ``get(name, shape, dtype)`` (plain tensors) and
        ``fp8w(name, shape)`` (e4m3 codes with 128x128 block scales), in Hugging Face
        DeepSeek-V3 names.  Experts are sharded expert parallel."""
        if not cfg.mla:
            raise ValueError("MLAWeights needs an MLA config")
        dev = torch.device(device)
        H, Hh = cfg.hidden_size, cfg.num_heads
        qr, kr = cfg.q_lora_rank, cfg.kv_lora_rank
        nope, rdim, vd = cfg.qk_nope_head_dim, cfg.qk_rope_head_dim, cfg.v_head_dim
        if kr != 512 or rdim != 64 or nope != 128 or vd != 128:
            raise ValueError("the sm_100a MLA kernels need kv_lora 512, rope 64, nope 128, v 128")
        E = cfg.num_experts
        e0, el = ep.split(E)
        I, Ie = cfg.intermediate_size, cfg.moe_intermediate_size
        Is = Ie * max(1, cfg.n_shared_experts)
        bf = torch.bfloat16

        layers = []
        for li in range(num_layers if num_layers is not None else cfg.num_layers):
            p = f"model.layers.{li}."
            a = p + "self_attn."
            q_a = fp8w(a + "q_a_proj.weight", (qr, H))
            kv_a = pad_rows_fp8(fp8w(a + "kv_a_proj_with_mqa.weight", (kr + rdim, H)), _pad128(kr + rdim))
            qkv_a = pad_rows_fp8(cat_fp8([q_a, kv_a]), _pad128(qr + kr + rdim))
            kv_b = get(a + "kv_b_proj.weight", (Hh * (nope + vd), kr), bf).view(Hh, nope + vd, kr)
            L = MLALayerWeights(
                attn_norm=get(p + "input_layernorm.weight", (H,), bf),
                w_qkv_a=qkv_a,
                q_a_norm=get(a + "q_a_layernorm.weight", (qr,), bf),
                w_q_b=fp8w(a + "q_b_proj.weight", (Hh * (nope + rdim), qr)),
                kv_a_norm=get(a + "kv_a_layernorm.weight", (kr,), torch.float32),
                w_uk=kv_b[:, :nope, :].transpose(1, 2).reshape(Hh * kr, nope).contiguous(),
                w_uv=kv_b[:, nope:, :].reshape(Hh * vd, kr).contiguous(),
                w_o=fp8w(a + "o_proj.weight", (H, Hh * vd)),
                mlp_norm=get(p + "post_attention_layernorm.weight", (H,), bf),
            )
            m = p + "mlp."
            if li < cfg.first_k_dense or not cfg.is_moe:
                L.dense = True
                L.w_gate_up = cat_fp8([fp8w(m + "gate_proj.weight", (I, H)),
                                       fp8w(m + "up_proj.weight", (I, H))])
                L.w_down = fp8w(m + "down_proj.weight", (H, I))
            else:
                L.dense = False
                L.router = get(m + "gate.weight", (E, H), bf)
                L.router_bias = get(m + "gate.e_score_correction_bias", (E,), torch.float32)
                gu, dn = [], []
                for e in range(e0, e0 + el):
                    x = m + f"experts.{e}."
                    gu.append(fp8w(x + "gate_proj.weight", (Ie, H)))
                    gu.append(fp8w(x + "up_proj.weight", (Ie, H)))
                    dn.append(fp8w(x + "down_proj.weight", (H, Ie)))
                L.experts_gate_up = cat_fp8(gu) if gu else None
                L.experts_down = cat_fp8(dn) if dn else None
                if cfg.n_shared_experts:
                    s_ = m + "shared_experts."
                    L.shared_gate_up = cat_fp8([fp8w(s_ + "gate_proj.weight", (Is, H)),
                                                fp8w(s_ + "up_proj.weight", (Is, H))])
                    L.shared_down = fp8w(s_ + "down_proj.weight", (H, Is))
            layers.append(L)
        embed = get("model.embed_tokens.weight", (cfg.vocab_size, H), bf)
        name = "model.embed_tokens.weight" if cfg.tie_word_embeddings else "lm_head.weight"
        lm_head = get(name, (cfg.vocab_size, H), bf)
        return cls(cfg, ep, embed, layers, get("model.norm.weight", (H,), bf), lm_head, e0, el)

    def nbytes(self) -> int:
        n = 0
        stack = [self.embed, self.lm_head, self.final_norm]
        for L in self.layers:
            for v in L.__dict__.values():
                if isinstance(v, torch.Tensor):
                    stack.append(v)
                elif isinstance(v, tuple):
                    stack.extend(v)
        for t in stack:
            n += t.numel() * t.element_size()
        return n


class MLAModel:
    """Forward pass of one rank (data-parallel MLA attention, expert-parallel MoE)."""

    def __init__(self, weights: MLAWeights, device, comm=None, max_positions: int | None = None):
        self.w = weights
        self.cfg = cfg = weights.cfg
        self.ep = weights.ep
        self.device = torch.device(device)
        self.comm = comm
        self.heads = cfg.num_heads
        self.num_kv_local = 1
        self.latent_dim = mla.QK
        mp = max_positions or cfg.max_position_embeddings
        self.cos_sin = rope.rope_cos_sin_table(mp, cfg.qk_rope_head_dim, cfg.rope_theta, None,
                                               device=self.device)
        self.scale = mla.softmax_scale(cfg.qk_nope_head_dim + cfg.qk_rope_head_dim, cfg.rope_scaling)
        self.qr = cfg.q_lora_rank
        self.kr = cfg.kv_lora_rank
        self.mode = moe_ops.MODE_SIGMOID_GROUP if cfg.router == "sigmoid_group" else moe_ops.MODE_SOFTMAX
        self.route_scale = cfg.routed_scaling_factor if cfg.router == "sigmoid_group" else 1.0
        self._head_offsets: dict[int, torch.Tensor] = {}

    @property
    def num_layers(self) -> int:
        return len(self.w.layers)

    def decode_splits(self, bsz: int, max_pages: int, sm_count: int) -> int:
        return mla.decode_splits(bsz, max_pages * 64, self.heads, sm_count)

    def _offsets(self, T: int) -> torch.Tensor:
        o = self._head_offsets.get(T)
        if o is None:
            o = (torch.arange(self.heads + 1, dtype=torch.int32, device=self.device) * T)
            self._head_offsets[T] = o
        return o

    # ------------------------------------------------------------ blocks
    def attention(self, L: MLALayerWeights, xq: torch.Tensor, xs: torch.Tensor, h: torch.Tensor,
                  fb: ForwardBatch, cache: torch.Tensor) -> None:
        """``xq`` / ``xs``: the normalised input in e4m3 with 1x128 scales."""
        cfg = self.cfg
        T, Hh = xq.shape[0], self.heads
        eps = cfg.rms_norm_eps
        qkv_a = fp8.linear(xq, xs, *L.w_qkv_a)
        q_a = qkv_a[:, : self.qr]
        kv_a = qkv_a[:, self.qr:]
        _, qnq, qns = norm.rmsnorm_fp8(q_a, L.q_a_norm, eps,
                                       out=torch.empty((T, self.qr), dtype=h.dtype, device=h.device))
        q = fp8.linear(qnq, qns, *L.w_q_b)
        mla.kv_write(kv_a, L.kv_a_norm, eps, fb.positions, fb.slots, self.cos_sin, cache)
        q_nope, q_pe = mla.q_prep(q, fb.positions, self.cos_sin, Hh)
        offs = self._offsets(T)
        q_lat = moe_ops.grouped_linear(q_nope.view(Hh * T, -1), L.w_uk, offs, Hh, rows_hint=T)
        o_lat = torch.empty((Hh, T, mla.LAT), dtype=h.dtype, device=h.device)
        mla.attention(q_lat.view(Hh, T, mla.LAT).transpose(0, 1), q_pe, cache, fb.block_table,
                      fb.seq_lens, cu_q=None if fb.is_decode else fb.cu_q,
                      max_q_len=1 if fb.is_decode else fb.max_q_len, scale=self.scale,
                      num_splits=fb.decode_splits if fb.is_decode else 1,
                      out=o_lat.transpose(0, 1))
        v = moe_ops.grouped_linear(o_lat.view(Hh * T, mla.LAT), L.w_uv, offs, Hh, rows_hint=T)
        a = mla.heads_to_tokens(v, T, Hh)
        aq, as_ = fp8.quantize(a)
        fp8.linear(aq, as_, *L.w_o, epi=fp8.EPI_RESADD, residual=h, out=h)

    def dense_mlp(self, L: MLALayerWeights, xq: torch.Tensor, xs: torch.Tensor, h: torch.Tensor) -> None:
        act = fp8.linear(xq, xs, *L.w_gate_up, epi=fp8.EPI_SWIGLU)
        aq, as_ = fp8.quantize(act)
        fp8.linear(aq, as_, *L.w_down, epi=fp8.EPI_RESADD, residual=h, out=h)

    def _shared(self, L: MLALayerWeights, xq: torch.Tensor, xs: torch.Tensor, h: torch.Tensor) -> None:
        if L.shared_gate_up is not None:
            sa = fp8.linear(xq, xs, *L.shared_gate_up, epi=fp8.EPI_SWIGLU)
            sq, ss = fp8.quantize(sa)
            fp8.linear(sq, ss, *L.shared_down, epi=fp8.EPI_RESADD, residual=h, out=h)

    def _moe_fused(self, L: MLALayerWeights, x: torch.Tensor, xq, xs, h: torch.Tensor, epc) -> None:
        """Decode MoE over peer memory: local routing, e4m3 dispatch to the expert owners,
        grouped GEMMs, combine fused into the down projection (``parallel/fused_ep.py``)."""
        cfg = self.cfg
        k = cfg.num_experts_per_tok
        e0, el = self.w.expert_start, self.w.experts_local
        T = x.shape[0]
        logits = gemm.linear(x, L.router, fp32_out=True)
        ids, wts = moe_ops.route(logits, k, mode=self.mode, renorm=cfg.norm_topk_prob,
                                 bias=L.router_bias, n_group=cfg.n_group, topk_group=cfg.topk_group,
                                 scale=self.route_scale)
        epc.dispatch(x, ids, wts, e0, el)
        local_ids = epc.recv_map(T, e0, el)
        offsets, pos, _ = moe_ops.permute(local_ids, el + 1)
        xpq, xps, inv = epc.gather(pos, offsets, T, e0, el)
        hint = max(1, (local_ids.numel() + cfg.num_experts - 1) // cfg.num_experts)
        act = fp8.grouped_linear(xpq, xps, *L.experts_gate_up, offsets, el, swiglu=True,
                                 rows_hint=hint)
        aq, as_ = fp8.quantize(act)
        epc.down_scatter(aq, as_, *L.experts_down, offsets, el, hint, inv, T, e0)
        self._shared(L, xq, xs, h)
        epc.combine(h, e0, el)

    def moe(self, L: MLALayerWeights, x: torch.Tensor, xq: torch.Tensor, xs: torch.Tensor,
            h: torch.Tensor) -> None:
        cfg = self.cfg
        k = cfg.num_experts_per_tok
        e0, el = self.w.expert_start, self.w.experts_local
        ep = self.ep.size
        epc = getattr(self.comm, "ep_fused", None) if ep > 1 else None
        if epc is not None and epc.fits(x.shape[0]):
            return self._moe_fused(L, x, xq, xs, h, epc)
        xa = self.comm.all_gather(x).view(-1, x.shape[1]) if ep > 1 else x
        Ta = xa.shape[0]
        logits = gemm.linear(xa, L.router, fp32_out=True)
        ids, wts = moe_ops.route(logits, k, mode=self.mode, renorm=cfg.norm_topk_prob,
                                 bias=L.router_bias, n_group=cfg.n_group, topk_group=cfg.topk_group,
                                 scale=self.route_scale)
        if ep > 1:
            local = ids - e0
            ids = torch.where((local >= 0) & (local < el), local, torch.full_like(local, el))
        offsets, rows, _ = moe_ops.permute(ids, el + 1)
        xp = moe_ops.gather(xa, rows, k)
        hint = max(1, (Ta * k + cfg.num_experts - 1) // cfg.num_experts)
        xpq, xps = fp8.quantize(xp)
        act = fp8.grouped_linear(xpq, xps, *L.experts_gate_up, offsets, el, swiglu=True, rows_hint=hint)
        aq, as_ = fp8.quantize(act)
        y = fp8.grouped_linear(aq, as_, *L.experts_down, offsets, el, rows_hint=hint)
        limit = offsets[el:el + 1]
        self._shared(L, xq, xs, h)
        if ep == 1:
            moe_ops.combine(y, rows, wts, k, residual=h, out=h, row_limit=limit)
            return
        part = moe_ops.combine(y, rows, wts, k, row_limit=limit)
        h.add_(self.comm.reduce_scatter(part))

    # ------------------------------------------------------------ forward
    def forward_hidden(self, fb: ForwardBatch, kv, h: torch.Tensor | None = None) -> torch.Tensor:
        cfg = self.cfg
        if h is None:
            h = sampling.embedding(fb.ids, self.w.embed)
        x = torch.empty_like(h)
        for li, L in enumerate(self.w.layers):
            cache, _ = kv.layer(li)
            # RMSNorm emits the e4m3 / 1x128 activation the fp8 GEMMs read in the same pass.
            _, xq, xs = norm.rmsnorm_fp8(h, L.attn_norm, cfg.rms_norm_eps, out=x)
            self.attention(L, xq, xs, h, fb, cache)
            _, xq, xs = norm.rmsnorm_fp8(h, L.mlp_norm, cfg.rms_norm_eps, out=x)
            if L.dense:
                self.dense_mlp(L, xq, xs, h)
            else:
                self.moe(L, x, xq, xs, h)
        return h

    def logits(self, h: torch.Tensor, fb: ForwardBatch) -> torch.Tensor:
        hl = h.index_select(0, fb.last_idx) if h.shape[0] != fb.last_idx.shape[0] else h
        x = norm.rmsnorm(hl, self.w.final_norm, self.cfg.rms_norm_eps)
        return gemm.linear(x, self.w.lm_head, fp32_out=True)

    def greedy(self, logits: torch.Tensor) -> torch.Tensor:
        return sampling.argmax(logits)

    def forward(self, fb: ForwardBatch, kv) -> torch.Tensor:
        return self.greedy(self.logits(self.forward_hidden(fb, kv), fb))


# ---------------------------------------------------------------------------- oracle
class MLAReference:
    """fp32 PyTorch oracle of the same network in the textbook (non-absorbed) form:
    per-head keys ``[k_nope = W_UK c_kv | k_pe]`` and values ``W_UV c_kv``, full
    recompute over the whole sequence.  Uses the dequantised fp8 weights, so the
    comparison isolates kernel numerics from quantisation."""

    def __init__(self, w: MLAWeights):
        if w.ep.size != 1:
            raise ValueError("the oracle runs unsharded weights")
        self.w = w
        self.cfg = w.cfg

    @staticmethod
    def _deq(wq: FP8) -> torch.Tensor:
        return fp8.dequantize(wq[0], wq[1], 128)

    @staticmethod
    def _lin_q(x: torch.Tensor, wq: FP8) -> torch.Tensor:
        """Linear with the activation quantised 1x128 like the kernels do."""
        xq, xs = fp8.quantize(x.to(torch.bfloat16).contiguous())
        return fp8.dequantize(xq, xs, 1) @ MLAReference._deq(wq).T

    def forward_logits(self, ids: torch.Tensor) -> torch.Tensor:
        cfg, w = self.cfg, self.w
        dev = w.embed.device
        T = ids.shape[0]
        Hh, nope, rdim, vd = cfg.num_heads, cfg.qk_nope_head_dim, cfg.qk_rope_head_dim, cfg.v_head_dim
        qr, kr = cfg.q_lora_rank, cfg.kv_lora_rank
        eps = cfg.rms_norm_eps
        pos = torch.arange(T, device=dev, dtype=torch.int32)
        cs = rope.rope_cos_sin_table(T + 1, rdim, cfg.rope_theta, None, device=dev)
        scale = mla.softmax_scale(nope + rdim, cfg.rope_scaling)
        h = w.embed[ids].float()

        def rms(v, g):
            return v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + eps) * g.float()

        for li, L in enumerate(w.layers):
            x = rms(h, L.attn_norm)
            qkv_a = self._lin_q(x, L.w_qkv_a)
            q = self._lin_q(rms(qkv_a[:, :qr], L.q_a_norm), L.w_q_b).view(T, Hh, nope + rdim)
            c = rms(qkv_a[:, qr:qr + kr], L.kv_a_norm)
            k_pe = mla.rope_interleaved_reference(qkv_a[:, qr + kr:qr + kr + rdim], pos, cs)
            q_pe = mla.rope_interleaved_reference(q[:, :, nope:], pos, cs)
            w_uk = L.w_uk.float().view(Hh, kr, nope)          # [h, latent, nope]
            w_uv = L.w_uv.float().view(Hh, vd, kr)
            k_nope = torch.einsum("tc,hcd->thd", c, w_uk)
            v = torch.einsum("tc,hvc->thv", c, w_uv)
            s = (torch.einsum("qhd,khd->hqk", q[:, :, :nope], k_nope)
                 + torch.einsum("qhd,kd->hqk", q_pe, k_pe)) * scale
            mask = torch.arange(T, device=dev)[None, :] > torch.arange(T, device=dev)[:, None]
            p = torch.softmax(s.masked_fill(mask[None], float("-inf")), dim=-1)
            o = torch.einsum("hqk,khv->qhv", p, v).reshape(T, Hh * vd)
            h = h + self._lin_q(o, L.w_o)
            x = rms(h, L.mlp_norm)
            if L.dense:
                gu = self._lin_q(x, L.w_gate_up)
                I = gu.shape[1] // 2
                h = h + self._lin_q(torch.nn.functional.silu(gu[:, :I]) * gu[:, I:], L.w_down)
                continue
            logits = x.to(torch.bfloat16).float() @ L.router.float().T
            ids_k, wts = moe_ops.route_reference(logits, cfg.num_experts_per_tok, mode=moe_ops.MODE_SIGMOID_GROUP
                                                 if cfg.router == "sigmoid_group" else moe_ops.MODE_SOFTMAX,
                                                 renorm=cfg.norm_topk_prob, bias=L.router_bias,
                                                 n_group=cfg.n_group, topk_group=cfg.topk_group,
                                                 scale=cfg.routed_scaling_factor
                                                 if cfg.router == "sigmoid_group" else 1.0)
            Ie = cfg.moe_intermediate_size
            H = cfg.hidden_size
            gu_all = self._deq(L.experts_gate_up).view(-1, 2 * Ie, H)
            dn_all = self._deq(L.experts_down).view(-1, H, Ie)
            y = torch.zeros_like(h)
            xq, xs = fp8.quantize(x.to(torch.bfloat16).contiguous())
            xd = fp8.dequantize(xq, xs, 1)
            for t in range(T):
                for j in range(ids_k.shape[1]):
                    e = int(ids_k[t, j])
                    g = xd[t] @ gu_all[e].T
                    a = (torch.nn.functional.silu(g[:Ie]) * g[Ie:]).to(torch.bfloat16)
                    aq, as_ = fp8.quantize(a[None].contiguous())
                    y[t] += wts[t, j] * (fp8.dequantize(aq, as_, 1)[0] @ dn_all[e].T)
            if L.shared_gate_up is not None:
                g = self._lin_q(x, L.shared_gate_up)
                Is = g.shape[1] // 2
                y = y + self._lin_q(torch.nn.functional.silu(g[:, :Is]) * g[:, Is:], L.shared_down)
            h = h + y
        x = rms(h, w.final_norm)
        return x.to(torch.bfloat16).float() @ w.lm_head.float().T

    def greedy(self, ids: list[int], n: int) -> list[int]:
        seq = list(ids)
        out = []
        for _ in range(n):
            logits = self.forward_logits(torch.tensor(seq, device=self.w.embed.device))
            tok = int(torch.argmax(logits[-1]))
            out.append(tok)
            seq.append(tok)
        return out
