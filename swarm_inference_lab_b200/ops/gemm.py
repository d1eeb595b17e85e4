"""tcgen05 GEMM entry points (``csrc/kernels/gemm_bf16.cu``).

``linear(x, w)`` computes ``x @ w.T`` in bf16 with fp32 accumulation.  The
epilogue variants fuse the work that follows a projection in a decoder layer:
residual add (attention output and down projections), SwiGLU (fused
``[gate; up]`` weight) and fp32 logits (LM head).
"""
from __future__ import annotations

import torch

from ._ext import ext
from .workspace import get_workspace

EPI_BF16 = 0
EPI_RESADD = 1
EPI_SWIGLU = 2
EPI_F32 = 3


def linear(x: torch.Tensor, w: torch.Tensor, *, out: torch.Tensor | None = None,
           residual: torch.Tensor | None = None, swiglu: bool = False, fp32_out: bool = False,
           force_mode: int = 0, force_splits: int = 0) -> torch.Tensor:
    """``epilogue(x @ w.T)``.

    * ``residual`` given: ``out = x @ w.T + residual`` (``out`` may alias ``residual``).
    * ``swiglu``: ``w = [gate; up]`` of shape ``[2*I, K]``; returns ``silu(x@gate.T) * (x@up.T)``.
    * ``fp32_out``: fp32 result (logits).
    ``force_mode`` 1/2 pins the swapped (decode) / normal (prefill) operand order, for tests.
    """
    if x.dim() != 2:
        x = x.reshape(-1, x.shape[-1])
    T = x.shape[0]
    n_out = w.shape[0] // 2 if swiglu else w.shape[0]
    if residual is not None:
        epi = EPI_RESADD
    elif swiglu:
        epi = EPI_SWIGLU
    elif fp32_out:
        epi = EPI_F32
    else:
        epi = EPI_BF16
    if out is None:
        dtype = torch.float32 if fp32_out else torch.bfloat16
        out = torch.empty((T, n_out), dtype=dtype, device=x.device)
    ws = get_workspace(x.device)
    ext().gemm_bf16(x, w, out, residual, epi, ws.ws, ws.counters, ws.status, force_mode,
                    force_splits)
    return out
