"""MXFP4 block quantisation and the SiTU-GLU activation: a CPU / PyTorch oracle.

MXFP4 (OCP Microscaling formats, v1.0): a block of 32 consecutive elements along the reduction
dimension shares one E8M0 scale (an 8-bit power of two, 2^(s - 127)); every element is an FP4
E2M1 code (sign, 2 exponent bits, 1 mantissa bit: magnitudes 0, 0.5, 1, 1.5, 2, 3, 4, 6).
Quantising a block follows the specification's rule: the shared exponent is
floor(log2(max |x|)) - 2 (2 being E2M1's largest exponent), each element x / 2^e is rounded to
the nearest E2M1 value (ties to the even code) and saturates at +-6.

Packing used here: ``packed[o, k // 2]`` holds element 2j in its low nibble and 2j + 1 in its
high nibble; ``scales[o, k // 32]`` is the biased exponent.  ``mxfp4_matmul`` computes
``x @ dequantise(packed, scales).T`` in fp32 -- the oracle a native (tcgen05 ``kind::mxf4``)
kernel would be checked against.

SiTU-GLU (the gated activation of the Kimi-K3-shaped fixture):
``gate = beta1 * tanh(g / beta1) * sigmoid(g) * beta2 * tanh(u / beta2)``, with the sigmoid
evaluated in the form that does not overflow for large |g|.

Reference: integrations/colibri/adapter/kimi_mxfp4_runtime.c:29-52 (MXFP4 matmul ABI; the
kernel itself lives in the external Colibri header, absent from the tree) and :118-140
(SiTU-GLU).
"""
from __future__ import annotations

import torch

BLOCK = 32
E2M1_MAX = 6.0
# magnitudes of the 8 non-negative E2M1 codes, code = index (sign in bit 3)
E2M1_VALUES = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def _round_e2m1(y: torch.Tensor) -> torch.Tensor:
    """Codes (0..15) of y rounded to the nearest E2M1 value, ties to the even code,
    saturating at +-6."""
    mag = y.abs().clamp(max=E2M1_MAX)
    vals = E2M1_VALUES.to(y.device)
    d = (mag.unsqueeze(-1) - vals).abs()
    best = d.min(dim=-1, keepdim=True).values
    ties = (d == best)
    # lowest index among the nearest, then prefer the even code of a tie
    idx = ties.float().argmax(dim=-1)
    two = ties.sum(-1) > 1
    if two.any():
        alt = (idx + 1).clamp(max=7)
        idx = torch.where(two & (idx % 2 == 1), alt, idx)
    sign = (y < 0) & (idx > 0)
    return (idx + 8 * sign.long()).to(torch.uint8)


def mxfp4_quantize(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """w [O, K] (K a multiple of 32) -> (packed uint8 [O, K/2], scales uint8 [O, K/32])."""
    if w.dim() != 2 or w.shape[1] % BLOCK:
        raise ValueError("mxfp4_quantize: w must be [O, K] with K a multiple of 32")
    O, K = w.shape
    blocks = w.float().reshape(O, K // BLOCK, BLOCK)
    amax = blocks.abs().amax(-1)
    e = torch.where(amax > 0, torch.floor(torch.log2(amax.clamp(min=1e-38))) - 2,
                    torch.full_like(amax, -127.0)).clamp(-127, 127)
    scales = (e + 127).to(torch.uint8)
    codes = _round_e2m1(blocks / torch.exp2(e).unsqueeze(-1)).reshape(O, K)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).to(torch.uint8)
    return packed, scales


def mxfp4_dequantize(packed: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """(packed [O, K/2], scales [O, K/32]) -> fp32 [O, K]."""
    O = packed.shape[0]
    lo = (packed & 0x0F).long()
    hi = (packed >> 4).long()
    codes = torch.stack([lo, hi], dim=-1).reshape(O, -1)
    vals = E2M1_VALUES.to(packed.device)[codes & 7] * torch.where(codes >= 8, -1.0, 1.0)
    K = codes.shape[1]
    scale = torch.exp2(scales.float() - 127).repeat_interleave(BLOCK, dim=1)[:, :K]
    return vals * scale


def mxfp4_matmul(x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """x [B, K] @ dequantise(packed, scales).T -> fp32 [B, O]."""
    return x.float() @ mxfp4_dequantize(packed, scales).T


def situ_glu(gate: torch.Tensor, up: torch.Tensor, beta1: float, beta2: float) -> torch.Tensor:
    """beta1 * tanh(g / beta1) * sigmoid(g) * beta2 * tanh(u / beta2) (fp32)."""
    if beta1 <= 0 or beta2 <= 0:
        raise ValueError("situ_glu: beta1 and beta2 must be positive")
    g, u = gate.float(), up.float()
    e = torch.exp(-g.abs())
    sig = torch.where(g >= 0, 1.0 / (1.0 + e), e / (1.0 + e))
    return beta1 * torch.tanh(g / beta1) * sig * beta2 * torch.tanh(u / beta2)
