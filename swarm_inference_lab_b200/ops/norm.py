"""RMSNorm kernels (``csrc/kernels/elementwise.cu``)."""
from __future__ import annotations

import torch

from ._ext import ext


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, *, out: torch.Tensor | None = None,
            residual: torch.Tensor | None = None,
            residual_out: torch.Tensor | None = None) -> torch.Tensor:
    """``out = rmsnorm(x [+ residual]) * weight``; with ``residual`` the sum is written to
    ``residual_out`` (defaults to ``residual`` itself, i.e. an in-place residual update)."""
    if out is None:
        out = torch.empty_like(x)
    if residual is not None and residual_out is None:
        residual_out = residual
    ext().rmsnorm(x, residual, residual_out, weight, out, float(eps), None, None)
    return out


def rmsnorm_fp8(x: torch.Tensor, weight: torch.Tensor, eps: float, *, out: torch.Tensor | None = None,
                residual: torch.Tensor | None = None, residual_out: torch.Tensor | None = None):
    """``rmsnorm`` that also emits the normalised rows quantised to e4m3 with one fp32
    scale per 1x128 block (the input format of the block-scaled fp8 GEMMs) in the same
    pass.  Returns (bf16 out, e4m3 codes uint8 [T, H], scales [T, H/128])."""
    T, H = x.shape
    if out is None:
        out = torch.empty((T, H), dtype=x.dtype, device=x.device)
    if residual is not None and residual_out is None:
        residual_out = residual
    q = torch.empty((T, H), dtype=torch.uint8, device=x.device)
    s = torch.empty((T, H // 128), dtype=torch.float32, device=x.device)
    ext().rmsnorm(x, residual, residual_out, weight, out, float(eps), q, s)
    return out, q, s


def rmsnorm_reference(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """HF-style RMSNorm in plain PyTorch (fp32 variance, bf16-rounded normalised value)."""
    dt = x.dtype
    xf = x.float()
    var = xf.pow(2).mean(-1, keepdim=True)
    return weight * (xf * torch.rsqrt(var + eps)).to(dt)
