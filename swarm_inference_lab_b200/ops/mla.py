"""Multi-head latent attention (DeepSeek-V3 / Kimi-K2) kernels (``csrc/kernels/mla.cu``).

Latent cache per layer: ``[num_pages, 64, 576]`` bf16 = RMS-normed ``c_kv`` (512)
followed by the rotated shared rope key ``k_pe`` (64, interleaved pairs).
Attention is computed in the weight-absorbed form (queries projected into the
512-wide latent space), so decode and prefill share one kernel.
"""
from __future__ import annotations

import math

import torch

from ._ext import ext
from .workspace import get_workspace

LAT, ROPE, QK = 512, 64, 576
PAGE_SIZE = 64


def softmax_scale(qk_head_dim: int, rope_scaling: dict | None = None) -> float:
    """``qk_head_dim ** -0.5``, times ``mscale ** 2`` under YaRN scaling (DeepSeek-V3)."""
    s = qk_head_dim ** -0.5
    if rope_scaling and rope_scaling.get("type", rope_scaling.get("rope_type")) == "yarn":
        factor = float(rope_scaling.get("factor", 1.0))
        mall = float(rope_scaling.get("mscale_all_dim", 0.0))
        if mall and factor > 1:
            m = 0.1 * mall * math.log(factor) + 1.0
            s *= m * m
    return s


def decode_splits(batch: int, max_ctx: int, heads: int = 64, sm_count: int = 148) -> int:
    """Split-KV factor: one wave of CTAs (one CTA per SM), >= 2 key tiles per split; the
    partials are merged by a separate, fully parallel kernel."""
    rb = max(1, (heads + 63) // 64)
    base = batch * rb
    want = max(1, sm_count // base)
    tiles = max(1, (max_ctx + 31) // 32)
    return int(max(1, min(want, tiles // 2, 64)))


def kv_write(kv_a: torch.Tensor, norm_w: torch.Tensor, eps: float, positions: torch.Tensor,
             slots: torch.Tensor, cos_sin: torch.Tensor, cache: torch.Tensor) -> None:
    """kv_a ``[T, >=576]`` (c_kv | k_pe) -> latent cache rows at ``slots``."""
    ext().mla_kv_write(kv_a, norm_w, float(eps), positions, slots, cos_sin, cache)


def q_prep(q: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor, heads: int):
    """q ``[T, H*192]`` -> (q_nope head-major ``[H, T, 128]``, rotated q_pe ``[T, H, 64]``)."""
    T = q.shape[0]
    q_nope = torch.empty((heads, T, 128), dtype=q.dtype, device=q.device)
    q_pe = torch.empty((T, heads, ROPE), dtype=q.dtype, device=q.device)
    ext().mla_q_prep(q, positions, cos_sin, q_nope, q_pe, heads)
    return q_nope, q_pe


def attention(q_lat: torch.Tensor, q_pe: torch.Tensor, cache: torch.Tensor,
              block_table: torch.Tensor, seq_lens: torch.Tensor, *, cu_q: torch.Tensor | None = None,
              max_q_len: int = 1, scale: float, num_splits: int = 1,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """q_lat ``[T, H, 512]`` and q_pe ``[T, H, 64]`` (any token/head strides) -> o_lat.

    ``cu_q`` None: one query per sequence (decode, T == B).  Otherwise packed
    queries with offsets ``cu_q`` [B+1] sitting at the end of each context."""
    if out is None:
        out = torch.empty((q_lat.shape[0], q_lat.shape[1], LAT), dtype=q_lat.dtype, device=q_lat.device)
    ws = get_workspace(q_lat.device)
    ext().mla_attention(q_lat, q_pe, cache, block_table, seq_lens, cu_q, out, float(scale),
                        int(max_q_len), int(num_splits), ws.attn_ws, ws.attn_counters, ws.status)
    return out


def heads_to_tokens(src: torch.Tensor, T: int, H: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """``[H, T, 128]`` -> ``[T, H*128]``."""
    if out is None:
        out = torch.empty((T, H * 128), dtype=src.dtype, device=src.device)
    ext().mla_heads_to_tokens(src, out, T, H)
    return out


# ------------------------------------------------------------------ references
def rope_interleaved_reference(x: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor):
    """Rotate pairs (2i, 2i+1) by frequency i.  x: [..., T, 64] with T leading after batch dims."""
    cs = cos_sin[positions.long()].to(x.device).float()
    d = x.shape[-1]
    cos, sin = cs[..., : d // 2], cs[..., d // 2:]
    while cos.dim() < x.dim():
        cos, sin = cos.unsqueeze(-2), sin.unsqueeze(-2)
    xf = x.float()
    x0, x1 = xf[..., 0::2], xf[..., 1::2]
    out = torch.empty_like(xf)
    out[..., 0::2] = x0 * cos - x1 * sin
    out[..., 1::2] = x1 * cos + x0 * sin
    return out


def attention_reference(q_lat: torch.Tensor, q_pe: torch.Tensor, lat: torch.Tensor, causal_offset: int,
                        scale: float) -> torch.Tensor:
    """fp32 absorbed MLA for one sequence.  q_lat [Tq, H, 512], q_pe [Tq, H, 64],
    lat [Tk, 576] (cache rows); query i sits at position causal_offset + i."""
    Tq = q_lat.shape[0]
    Tk = lat.shape[0]
    q = torch.cat([q_lat.float(), q_pe.float()], dim=-1)
    s = torch.einsum("qhd,kd->hqk", q, lat.float()) * scale
    qpos = torch.arange(Tq, device=q.device)[:, None] + causal_offset
    kpos = torch.arange(Tk, device=q.device)[None, :]
    s = s.masked_fill((kpos > qpos)[None], float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("hqk,kd->qhd", p, lat[:, :LAT].float())
