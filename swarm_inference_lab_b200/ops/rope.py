"""Rotary position embedding tables and the fused q/k-norm + RoPE + paged KV write."""
from __future__ import annotations

import math

import torch

from ._ext import ext


def rope_inv_freq(head_dim: int, theta: float, scaling: dict | None = None) -> torch.Tensor:
    """Inverse frequencies in float64, with optional Llama-3 style frequency scaling."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    if scaling and scaling.get("rope_type", scaling.get("type")) == "llama3":
        factor = float(scaling["factor"])
        low = float(scaling.get("low_freq_factor", 1.0))
        high = float(scaling.get("high_freq_factor", 4.0))
        old_ctx = float(scaling.get("original_max_position_embeddings", 8192))
        low_wl, high_wl = old_ctx / low, old_ctx / high
        wl = 2 * math.pi / inv
        scaled = torch.where(wl > low_wl, inv / factor, inv)
        smooth = (old_ctx / wl - low) / (high - low)
        mid = (1 - smooth) * scaled / factor + smooth * scaled
        is_mid = (wl >= high_wl) & (wl <= low_wl)
        inv = torch.where(is_mid, mid, scaled)
    return inv


def rope_cos_sin_table(max_pos: int, head_dim: int, theta: float, scaling: dict | None = None,
                       device=None) -> torch.Tensor:
    """``[max_pos, head_dim]`` fp32: first half cos, second half sin (rotate-half form)."""
    inv = rope_inv_freq(head_dim, theta, scaling)
    pos = torch.arange(max_pos, dtype=torch.float64)
    ang = torch.outer(pos, inv)
    tab = torch.cat([ang.cos(), ang.sin()], dim=-1).to(torch.float32)
    return tab.to(device) if device is not None else tab


def rope_kv_write(qkv: torch.Tensor, positions: torch.Tensor, slots: torch.Tensor,
                  cos_sin: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                  num_q_heads: int, num_kv_heads: int, q_norm: torch.Tensor | None = None,
                  k_norm: torch.Tensor | None = None, eps: float = 1e-6) -> None:
    """Rotate the q heads of ``qkv`` in place and write rotated k and raw v to the cache."""
    ext().rope_kv_write(qkv, positions, slots, cos_sin, q_norm, k_norm, float(eps), k_cache,
                        v_cache, num_q_heads, num_kv_heads)


def apply_rope_reference(x: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor) -> torch.Tensor:
    """Rotate-half RoPE in plain PyTorch.  x: [T, H, D]."""
    d = x.shape[-1]
    cs = cos_sin[positions.long()].to(x.device)
    cos, sin = cs[:, None, : d // 2], cs[:, None, d // 2:]
    xf = x.float()
    x1, x2 = xf[..., : d // 2], xf[..., d // 2:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1).to(x.dtype)
