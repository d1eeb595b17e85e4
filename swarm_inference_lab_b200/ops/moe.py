"""Mixture-of-experts ops on the sm_100a kernels (``csrc/kernels/moe.cu`` and the
grouped tcgen05 GEMM), plus their plain-PyTorch references.

Pipeline of one MoE MLP on a rank that owns experts [e0, e0+E_local):

    router logits (tcgen05 GEMM, fp32) -> moe_topk -> moe_permute (counts,
    offsets, rows) -> moe_gather (expert-sorted rows) -> grouped GEMM with the
    SwiGLU epilogue (gate/up) -> grouped GEMM (down) -> moe_combine
    (weighted, slot-ordered sum + residual [+ shared expert]).
"""
from __future__ import annotations

import torch

from ._ext import ext
from . import gemm
from .workspace import get_workspace

MODE_SOFTMAX = 0
MODE_SIGMOID_GROUP = 1


def route(logits: torch.Tensor, k: int, *, mode: int = MODE_SOFTMAX, renorm: bool = True,
          bias: torch.Tensor | None = None, n_group: int = 1, topk_group: int = 1,
          scale: float = 1.0):
    T = logits.shape[0]
    ids = torch.empty((T, k), dtype=torch.int32, device=logits.device)
    w = torch.empty((T, k), dtype=torch.float32, device=logits.device)
    ext().moe_topk(logits.contiguous(), k, mode, renorm, bias, n_group, topk_group, float(scale),
                   ids, w)
    return ids, w


def permute(ids: torch.Tensor, num_experts: int):
    offsets = torch.empty(num_experts + 1, dtype=torch.int32, device=ids.device)
    rows = torch.empty(ids.numel(), dtype=torch.int32, device=ids.device)
    counts = torch.empty(num_experts, dtype=torch.int32, device=ids.device)
    ext().moe_permute(ids.reshape(-1).contiguous(), num_experts, offsets, rows, counts)
    return offsets, rows, counts


def gather(x: torch.Tensor, rows: torch.Tensor, k: int, out: torch.Tensor | None = None):
    if out is None:
        out = torch.empty((rows.numel(), x.shape[1]), dtype=x.dtype, device=x.device)
    ext().moe_gather(x, rows, k, out)
    return out


def grouped_linear(xp: torch.Tensor, w: torch.Tensor, offsets: torch.Tensor, num_groups: int, *,
                   swiglu: bool = False, rows_hint: int = 16, out: torch.Tensor | None = None):
    rows_per = w.shape[0] // num_groups
    n_out = rows_per // 2 if swiglu else rows_per
    if out is None:
        out = torch.empty((xp.shape[0], n_out), dtype=torch.bfloat16, device=xp.device)
    ws = get_workspace(xp.device)
    ext().gemm_grouped(xp, w, out, offsets, num_groups, swiglu, int(rows_hint), ws.ws,
                       ws.counters, ws.status)
    return out


def combine(y: torch.Tensor, rows: torch.Tensor, weights: torch.Tensor, k: int, *,
            residual: torch.Tensor | None = None, shared: torch.Tensor | None = None,
            out: torch.Tensor | None = None, row_limit: torch.Tensor | None = None) -> torch.Tensor:
    """``out[t] = residual[t] + shared[t] + sum_s w[t,s] * y[rows[t,s]]``; assignments whose
    row is >= ``row_limit[0]`` (experts owned by other ranks) are skipped."""
    T = weights.shape[0]
    if out is None:
        out = torch.empty((T, y.shape[1]), dtype=torch.bfloat16, device=y.device)
    ext().moe_combine(y, rows, weights.contiguous(), k, residual, shared, out, row_limit)
    return out


def moe_mlp(x: torch.Tensor, router_w: torch.Tensor, w_gate_up: torch.Tensor,
            w_down: torch.Tensor, num_experts: int, k: int, *, mode: int = MODE_SOFTMAX,
            renorm: bool = True, bias: torch.Tensor | None = None, n_group: int = 1,
            topk_group: int = 1, scale: float = 1.0, residual: torch.Tensor | None = None,
            shared: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Full single-rank MoE MLP: returns ``residual + shared + sum_k w_k * expert_k(x)``."""
    T = x.shape[0]
    logits = gemm.linear(x, router_w, fp32_out=True)
    ids, w = route(logits, k, mode=mode, renorm=renorm, bias=bias, n_group=n_group,
                   topk_group=topk_group, scale=scale)
    offsets, rows, _ = permute(ids, num_experts)
    xp = gather(x, rows, k)
    hint = max(1, (T * k + num_experts - 1) // num_experts)
    act = grouped_linear(xp, w_gate_up, offsets, num_experts, swiglu=True, rows_hint=hint)
    y = grouped_linear(act, w_down, offsets, num_experts, rows_hint=hint)
    return combine(y, rows, w, k, residual=residual, shared=shared, out=out)


# ------------------------------------------------------------------ references
def route_reference(logits: torch.Tensor, k: int, *, mode: int = MODE_SOFTMAX, renorm: bool = True,
                    bias: torch.Tensor | None = None, n_group: int = 1, topk_group: int = 1,
                    scale: float = 1.0):
    """fp32 routing with lowest-id tie breaks (stable sort on descending keys)."""
    lf = logits.float()
    T, E = lf.shape
    if mode == MODE_SOFTMAX:
        score = torch.softmax(lf, dim=-1)
        key = score
    else:
        score = torch.sigmoid(lf)
        key = score + (bias.float() if bias is not None else 0.0)
        if n_group > 1:
            g = key.view(T, n_group, E // n_group)
            gs = g.topk(2, dim=-1).values.sum(-1)
            order = torch.sort(-gs, dim=-1, stable=True).indices[:, :topk_group]
            mask = torch.zeros(T, n_group, dtype=torch.bool, device=lf.device)
            mask.scatter_(1, order, True)
            key = key.masked_fill(~mask.repeat_interleave(E // n_group, dim=1), float("-inf"))
    ids = torch.sort(-key, dim=-1, stable=True).indices[:, :k]
    w = score.gather(1, ids)
    if renorm:
        w = w / w.sum(-1, keepdim=True)
    return ids.to(torch.int32), w * scale


def moe_mlp_reference(x, router_w, w_gate_up, w_down, num_experts, k, *, mode=MODE_SOFTMAX,
                      renorm=True, bias=None, n_group=1, topk_group=1, scale=1.0, residual=None,
                      shared=None):
    T, H = x.shape
    logits = x.float() @ router_w.float().T
    ids, w = route_reference(logits, k, mode=mode, renorm=renorm, bias=bias, n_group=n_group,
                             topk_group=topk_group, scale=scale)
    gu = w_gate_up.float().view(num_experts, -1, H)
    dn = w_down.float().view(num_experts, H, -1)
    inter = gu.shape[1] // 2
    out = torch.zeros(T, H, dtype=torch.float32, device=x.device)
    for s in range(k):
        e = ids[:, s].long()
        h = torch.einsum("th,tih->ti", x.float(), gu[e])
        a = torch.nn.functional.silu(h[:, :inter]) * h[:, inter:]
        a = a.to(torch.bfloat16).float()
        y = torch.einsum("ti,thi->th", a, dn[e]).to(torch.bfloat16).float()
        out += w[:, s:s + 1] * y
    if shared is not None:
        out += shared.float()
    if residual is not None:
        out += residual.float()
    return out.to(torch.bfloat16), ids, w
