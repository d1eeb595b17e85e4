"""Paged GQA attention kernels (``csrc/kernels/attention.cu``).

KV cache per layer: ``[num_pages, num_kv_heads, 64, 128]`` bf16 for K and V.
"""
from __future__ import annotations

import math
import os

import torch

from ._ext import ext
from .workspace import get_workspace

PAGE_SIZE = 64


def decode_splits(batch: int, kv_heads: int, max_pages: int, sm_count: int = 148) -> int:
    """Split-KV factor: about 256 (sequence, KV head) CTAs in total, at most 8 splits and at
    least 2 pages per split.  Two decode CTAs fit on an SM (3 page stages each), so 256 CTAs
    are one wave on 148 SMs; more splits only add partials for the last CTA to merge.
    Measured on B200 (2k context, graph-timed): 32 sequences x 8 KV heads run best unsplit
    (44.7 us, 0.92 of HBM, against 54.8 us with 4 splits); 32 x 1 KV head best with 8 splits
    (13.7 us); 1 sequence x 8 KV heads best with 8 (11.6 us, against 15.1 us with 16)."""
    del sm_count  # the 256-CTA target already encodes 2 CTAs on each of 148 SMs
    pairs = max(1, batch * kv_heads)
    cap = max(1, min(8, max_pages // 2))
    return int(max(1, min(cap, 256 // pairs)))


def paged_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                 block_table: torch.Tensor, seq_lens: torch.Tensor, *, out: torch.Tensor | None = None,
                 num_splits: int = 1, scale: float | None = None) -> torch.Tensor:
    """q: [B, Hq, 128] (one new token per sequence) -> out [B, Hq*128]."""
    B, Hq, D = q.shape
    if out is None:
        out = torch.empty((B, Hq * D), dtype=q.dtype, device=q.device)
    ws = get_workspace(q.device)
    ext().paged_decode(q, k_cache, v_cache, block_table, seq_lens, out,
                       scale if scale is not None else 1.0 / math.sqrt(D), int(num_splits),
                       ws.attn_ws, ws.attn_counters, ws.status)
    return out


PREFILL_KERNEL = os.environ.get("SIL_PREFILL_ATTN", "tc")  # tc (tcgen05) | mma (mma.sync)


def paged_prefill(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                  block_table: torch.Tensor, seq_lens: torch.Tensor, cu_q: torch.Tensor,
                  max_q_len: int, *, out: torch.Tensor | None = None,
                  scale: float | None = None, kernel: str | None = None) -> torch.Tensor:
    """q: packed [T, Hq, 128]; cu_q: [B+1] int32 query offsets -> out [T, Hq*128].

    ``kernel`` "tc" runs the tcgen05 kernel (S and O in TMEM, 128 queries x 128 keys per
    step); "mma" the earlier ``mma.sync`` kernel (64-query tiles).  Short query chunks (at
    most 16 queries per sequence: speculative verification, small chunks) use "mma"."""
    T, Hq, D = q.shape
    if out is None:
        out = torch.empty((T, Hq * D), dtype=q.dtype, device=q.device)
    ws = get_workspace(q.device)
    sc = scale if scale is not None else 1.0 / math.sqrt(D)
    kind = kernel or PREFILL_KERNEL
    if kind == "tc" and max_q_len > 16 and q.stride(0) % 8 == 0:
        ext().paged_prefill_tc(q, k_cache, v_cache, block_table, seq_lens, cu_q, out, sc,
                               int(max_q_len), ws.status)
    else:
        ext().paged_prefill(q, k_cache, v_cache, block_table, seq_lens, cu_q, out, sc,
                            int(max_q_len), ws.status)
    return out


def attention_reference(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal_offset: int,
                        scale: float | None = None) -> torch.Tensor:
    """Dense GQA attention in fp32.  q: [Tq, Hq, D], k/v: [Tk, Hkv, D]; query i sits at
    absolute position ``causal_offset + i`` and sees keys ``<=`` that position."""
    Tq, Hq, D = q.shape
    Tk, Hkv, _ = k.shape
    g = Hq // Hkv
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    kf = k.float().repeat_interleave(g, dim=1)
    vf = v.float().repeat_interleave(g, dim=1)
    s = torch.einsum("qhd,khd->hqk", q.float(), kf) * scale
    qpos = torch.arange(Tq, device=q.device)[:, None] + causal_offset
    kpos = torch.arange(Tk, device=q.device)[None, :]
    s = s.masked_fill((kpos > qpos)[None], float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("hqk,khd->qhd", p, vf)
