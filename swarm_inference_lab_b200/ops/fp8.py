"""Block-scaled fp8 (e4m3) linear layers: the DeepSeek-V3 / Kimi-K2 weight format.

Weights: e4m3 ``[N, K]`` with fp32 scales ``[N/128, K/128]`` (one per 128x128
block, ``w ~= q * s``).  Activations: bf16 rows quantised on the device to
e4m3 with one fp32 scale per 1x128 block (``quantize``).  ``linear`` runs the
tcgen05 kind::f8f6f4 GEMM with per-block promotion (``csrc/kernels/gemm_fp8.cu``).
"""
from __future__ import annotations

import torch

from ._ext import ext
from .workspace import get_workspace

EPI_BF16, EPI_RESADD, EPI_SWIGLU, EPI_F32 = 0, 1, 2, 3
E4M3_MAX = 448.0


def quantize(x: torch.Tensor):
    """bf16 [T, K] -> (e4m3 codes as uint8 [T, K], fp32 scales [T, K/128])."""
    T, K = x.shape
    q = torch.empty((T, K), dtype=torch.uint8, device=x.device)
    s = torch.empty((T, K // 128), dtype=torch.float32, device=x.device)
    ext().quant_fp8_1x128(x, q, s)
    return q, s


def quantize_weight(w: torch.Tensor):
    """fp32/bf16 [N, K] -> (e4m3 uint8 [N, K], fp32 block scales [N/128, K/128]) (torch ops)."""
    N, K = w.shape
    blocks = w.float().reshape(N // 128, 128, K // 128, 128)
    amax = blocks.abs().amax(dim=(1, 3)).clamp_min(1e-12)
    scale = amax / E4M3_MAX
    q = (blocks / scale[:, None, :, None]).clamp(-E4M3_MAX, E4M3_MAX)
    q = q.reshape(N, K).to(torch.float8_e4m3fn).view(torch.uint8)
    return q.contiguous(), scale.contiguous()


def dequantize(q: torch.Tensor, s: torch.Tensor, block_rows: int) -> torch.Tensor:
    """Inverse of the quantisers above (fp32)."""
    v = q.view(torch.float8_e4m3fn).float()
    sr = s.repeat_interleave(block_rows, dim=0)[: v.shape[0]] if block_rows > 1 else s
    return v * sr.repeat_interleave(128, dim=1)


def linear(xq, xs, wq, wscale, *, epi: int = EPI_BF16, residual=None, out=None):
    T = xq.shape[0]
    n_out = wq.shape[0] // 2 if epi == EPI_SWIGLU else wq.shape[0]
    if out is None:
        out = torch.empty((T, n_out), dtype=torch.float32 if epi == EPI_F32 else torch.bfloat16,
                          device=xq.device)
    ws = get_workspace(xq.device)
    ext().gemm_fp8(xq, xs, wq, wscale, out, residual, epi, ws.ws, ws.counters, ws.status)
    return out


def grouped_linear(xq, xs, wq, wscale, offsets, num_groups: int, *, swiglu: bool = False,
                   rows_hint: int = 16, out=None):
    rows = wq.shape[0] // num_groups
    n_out = rows // 2 if swiglu else rows
    if out is None:
        out = torch.empty((xq.shape[0], n_out), dtype=torch.bfloat16, device=xq.device)
    ws = get_workspace(xq.device)
    ext().gemm_fp8_grouped(xq, xs, wq, wscale, out, offsets, num_groups, swiglu, int(rows_hint),
                           ws.ws, ws.counters, ws.status)
    return out


def linear_reference(xq, xs, wq, wscale) -> torch.Tensor:
    """fp32 reference: per-block dequantised product."""
    x = dequantize(xq, xs, 1)
    w = dequantize(wq, wscale, 128)
    return x @ w.T
