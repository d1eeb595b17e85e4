"""Decode-step and single-kernel timing harness (CUDA events, no profiler).

    python -m swarm_inference_lab_b200.utils.profile_decode --batch 32 --ctx 2048 [--steps 5]
    python -m swarm_inference_lab_b200.utils.profile_decode --op gemm --m 28672 --n 32 --k 4096 --swiglu
    python -m swarm_inference_lab_b200.utils.profile_decode --op decode_attn --batch 32 --ctx 2048
    python -m swarm_inference_lab_b200.utils.profile_decode --op prefill_attn --batch 32 --ctx 2048 --kernel tc
    python -m swarm_inference_lab_b200.utils.profile_decode --op mla_decode --batch 32 --ctx 4096
    python -m swarm_inference_lab_b200.utils.profile_decode --op fp8_grouped --groups 48 --n 6 --m 7168 --k 2048
    python -m swarm_inference_lab_b200.utils.profile_decode --op prefill_gemms --n 65536 --layers 32

The decode mode builds the Llama-3-8B-shaped model with random weights and
a KV cache whose pages hold random values (attention cost depends only on
the context length), then runs eager decode steps: suitable for a kernel
launch list under ``ncu`` (each step issues the same launch sequence).
The op modes time one kernel on a small case and report achieved bytes/s
and FLOP/s against the measured box peaks.
"""
from __future__ import annotations

import argparse
import json
import os

import torch

PEAKS = {"hbm_gbs": 6534.1, "bf16_tflops": 1649.5}


def _peaks():
    p = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"]}
    except (OSError, KeyError, ValueError):
        return PEAKS


def time_fn(fn, iters: int = 20, warmup: int = 3, graph: bool = True) -> float:
    """Mean milliseconds per call.  With ``graph`` the calls are captured once into a
    CUDA graph and replayed, so host launch overhead is excluded (GPU time only)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    g = None
    if graph:
        s0 = torch.cuda.Stream()
        s0.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s0):
            fn()
        torch.cuda.current_stream().wait_stream(s0)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s0):
            for _ in range(iters):
                fn()
        g.replay()
        torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    if g is not None:
        g.replay()
    else:
        for _ in range(iters):
            fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def op_gemm(a):
    from ..ops import gemm
    T, N, K = a.n, a.m, a.k
    x = torch.randn(T, K, device="cuda").bfloat16()
    rows = 2 * N if a.swiglu else N
    w = (torch.randn(rows, K, device="cuda") * 0.02).bfloat16()
    ms = time_fn(lambda: gemm.linear(x, w, swiglu=a.swiglu, force_splits=a.splits), a.iters,
                 graph=not a.eager)
    bytes_ = rows * K * 2 + T * K * 2 + T * N * 2
    flops = 2 * T * rows * K
    pk = _peaks()
    return {"op": "gemm", "tokens": T, "out_features": N, "k": K, "swiglu": a.swiglu,
            "splits": a.splits or "auto", "ms": ms,
            "GBps": bytes_ / ms / 1e6, "TFLOPs": flops / ms / 1e9,
            "frac_hbm_of_measured": bytes_ / ms / 1e6 / pk["hbm_gbs"],
            "frac_bf16_of_measured": flops / ms / 1e9 / pk["bf16_tflops"]}


def op_decode_attn(a):
    from ..ops import attention as A
    B, ctx, hq, hkv = a.batch, a.ctx, a.hq, a.hkv
    pages_per = (ctx + 63) // 64
    P = B * pages_per
    kc = torch.randn(P, hkv, 64, 128, device="cuda").bfloat16()
    vc = torch.randn_like(kc)
    bt = torch.arange(P, dtype=torch.int32, device="cuda").view(B, pages_per)
    sl = torch.full((B,), ctx, dtype=torch.int32, device="cuda")
    q = torch.randn(B, hq, 128, device="cuda").bfloat16()
    splits = a.splits or A.decode_splits(B, hkv, pages_per)
    ms = time_fn(lambda: A.paged_decode(q, kc, vc, bt, sl, num_splits=splits), a.iters,
                 graph=not a.eager)
    bytes_ = 2 * B * ctx * hkv * 128 * 2
    pk = _peaks()
    return {"op": "paged_decode", "batch": B, "ctx": ctx, "splits": splits, "ms": ms,
            "GBps": bytes_ / ms / 1e6, "frac_hbm_of_measured": bytes_ / ms / 1e6 / pk["hbm_gbs"]}


def op_prefill_attn(a):
    """Causal paged prefill attention of ``batch`` sequences of ``ctx`` tokens (all new):
    the tcgen05 kernel or the mma.sync kernel (``--kernel``); FLOPs count the causal half."""
    from ..ops import attention as A
    B, ctx, hq, hkv = a.batch, a.ctx, a.hq, a.hkv
    pages_per = (ctx + 63) // 64
    P = B * pages_per
    kc = torch.randn(P, hkv, 64, 128, device="cuda").bfloat16()
    vc = torch.randn_like(kc)
    bt = torch.arange(P, dtype=torch.int32, device="cuda").view(B, pages_per)
    sl = torch.full((B,), ctx, dtype=torch.int32, device="cuda")
    T = B * ctx
    qkv = torch.randn(T, (hq + 2 * hkv) * 128, device="cuda").bfloat16()
    q = qkv.as_strided((T, hq, 128), (qkv.stride(0), 128, 1))
    cu = torch.arange(0, T + 1, ctx, dtype=torch.int32, device="cuda")
    out = torch.empty(T, hq * 128, device="cuda", dtype=torch.bfloat16)
    ms = time_fn(lambda: A.paged_prefill(q, kc, vc, bt, sl, cu, ctx, out=out, kernel=a.kernel),
                 a.iters, graph=not a.eager)
    flops = 4.0 * B * hq * 128 * ctx * (ctx + 1) / 2
    pk = _peaks()
    return {"op": "paged_prefill", "kernel": a.kernel, "batch": B, "ctx": ctx, "heads": hq,
            "ms": ms, "TFLOPs": flops / ms / 1e9,
            "frac_bf16_of_measured": flops / ms / 1e9 / pk["bf16_tflops"]}


def op_launch_floor(a):
    """Device time per launch of the smallest kernels in a captured graph (the per-kernel
    floor a decode step pays): a 1x128 RMSNorm and a 128x128x64 GEMM."""
    from ..ops import gemm, norm
    x = torch.randn(1, 128, device="cuda").bfloat16()
    wn = torch.ones(128, device="cuda").bfloat16()
    y = torch.empty_like(x)
    w = torch.randn(128, 64, device="cuda").bfloat16()
    xg = torch.randn(1, 64, device="cuda").bfloat16()
    return {"op": "launch_floor",
            "rmsnorm_us": 1e3 * time_fn(lambda: norm.rmsnorm(x, wn, 1e-6, out=y), a.iters),
            "gemm_tiny_us": 1e3 * time_fn(lambda: gemm.linear(xg, w), a.iters)}


def op_gemm_ar1(a):
    """The fused row-parallel GEMM + all-reduce kernel with a one-rank group (its own buffer
    as the only peer): the kernel's own cost without NVLink, next to the plain GEMM with the
    residual epilogue.  One GPU, so it can be profiled."""
    from ..ops import gemm
    from ..ops._ext import ext
    from ..ops.workspace import get_workspace
    T, N, K = a.n, a.m, a.k
    x = torch.randn(T, K, device="cuda").bfloat16()
    w = (torch.randn(N, K, device="cuda") * 0.02).bfloat16()
    h = torch.randn(T, N, device="cuda").bfloat16()
    max_tiles, max_tokens = (N + 127) // 128, 128
    flags_off = 256
    slots_off = ((flags_off + 2 * 8 * max_tiles * 4 + 255) // 256) * 256
    nbytes = slots_off + 2 * 8 * max_tokens * N * 2
    e = ext()
    buf = e.symm_alloc(nbytes, torch.cuda.current_device())
    ws = get_workspace()
    try:
        fused = time_fn(lambda: e.gemm_allreduce(x, w, h, [buf], 0, max_tiles, max_tokens, N, flags_off,
                                                 slots_off, ws.ws, ws.counters, ws.status),
                        a.iters, graph=not a.eager)
        plain = time_fn(lambda: gemm.linear(x, w, out=h, residual=h), a.iters, graph=not a.eager)
        ws.check()
    finally:
        torch.cuda.synchronize()
        e.symm_free(buf)
    bytes_ = N * K * 2
    pk = _peaks()
    return {"op": "gemm_allreduce_1rank", "tokens": T, "out": N, "k": K, "fused_ms": fused,
            "plain_residual_ms": plain, "weight_frac_hbm_fused": bytes_ / fused / 1e6 / pk["hbm_gbs"]}


def op_mla_decode(a):
    """Absorbed MLA decode over a [pages, 64, 576] latent cache, 64 heads."""
    from ..ops import mla
    B, ctx, H = a.batch, a.ctx, 64
    pages_per = (ctx + 63) // 64
    cache = torch.randn(B * pages_per, 64, 576, device="cuda").bfloat16()
    bt = torch.arange(B * pages_per, dtype=torch.int32, device="cuda").view(B, pages_per)
    sl = torch.full((B,), ctx, dtype=torch.int32, device="cuda")
    q_lat = torch.randn(B, H, 512, device="cuda").bfloat16()
    q_pe = torch.randn(B, H, 64, device="cuda").bfloat16()
    splits = mla.decode_splits(B, ctx, H)
    ms = time_fn(lambda: mla.attention(q_lat, q_pe, cache, bt, sl, scale=192 ** -0.5,
                                       num_splits=splits), a.iters, graph=not a.eager)
    bytes_ = B * ctx * 576 * 2
    flops = 2 * B * H * ctx * (576 + 512)
    pk = _peaks()
    return {"op": "mla_decode", "batch": B, "ctx": ctx, "heads": H, "splits": splits, "ms": ms,
            "GBps": bytes_ / ms / 1e6, "TFLOPs": flops / ms / 1e9,
            "frac_hbm_of_measured": bytes_ / ms / 1e6 / pk["hbm_gbs"],
            "frac_bf16_of_measured": flops / ms / 1e9 / pk["bf16_tflops"]}


def op_fp8_grouped(a):
    """Grouped block-scaled e4m3 GEMM (experts): ``groups`` x [m, k] weights, ``n`` rows each."""
    from ..ops import fp8
    G, rows, N, K = a.groups, a.n, a.m, a.k
    wq = torch.randint(0, 100, (G * N, K), dtype=torch.uint8, device="cuda")
    ws = torch.rand(G * N // 128, K // 128, device="cuda") * 1e-3
    x = torch.randn(G * rows, K, device="cuda").bfloat16()
    xq, xs = fp8.quantize(x)
    off = torch.arange(G + 1, dtype=torch.int32, device="cuda") * rows
    ms = time_fn(lambda: fp8.grouped_linear(xq, xs, wq, ws, off, G, rows_hint=rows), a.iters,
                 graph=not a.eager)
    bytes_ = G * N * K + G * rows * K + G * rows * N * 2
    flops = 2 * G * rows * N * K
    pk = _peaks()
    return {"op": "fp8_grouped", "groups": G, "rows_per_group": rows, "out": N, "k": K, "ms": ms,
            "GBps": bytes_ / ms / 1e6, "frac_hbm_of_measured": bytes_ / ms / 1e6 / pk["hbm_gbs"],
            "TFLOPs": flops / ms / 1e9}


def decode_steps(a):
    from ..engine.kv_cache import PagedKVCache
    from ..models.config import preset
    from ..models.dense import DenseModel, DenseWeights, ForwardBatch, TPInfo
    from ..ops import attention as A
    cfg = preset(a.model)
    if a.layers:
        cfg = cfg.replace(num_layers=a.layers)
    # --tp N: one rank's shard of an N-way tensor-parallel model with the all-reduces
    # left out (a local communicator), i.e. the compute part of a TP decode step.
    tp = TPInfo(0, a.tp)
    w = DenseWeights.random(cfg, tp, "cuda", seed=0)
    from ..parallel.comm import LocalComm
    model = DenseModel(w, "cuda", comm=LocalComm(), max_positions=a.ctx + 64)
    B = a.batch
    pages_per = (a.ctx + 1 + 63) // 64
    kvh = tp.heads(cfg.num_kv_heads)[1]
    kv = PagedKVCache(cfg.num_layers, kvh, B * pages_per, "cuda")
    kv.k.normal_()
    kv.v.normal_()
    bt = torch.arange(B * pages_per, dtype=torch.int32, device="cuda").view(B, pages_per)
    pos = torch.full((B,), a.ctx, dtype=torch.int32, device="cuda")
    slots = bt[:, a.ctx // 64] * 64 + a.ctx % 64
    fb = ForwardBatch(ids=torch.randint(0, cfg.vocab_size, (B,), device="cuda"), positions=pos,
                      slots=slots.int(), seq_lens=pos + 1, block_table=bt,
                      last_idx=torch.arange(B, device="cuda"), is_decode=True,
                      decode_splits=A.decode_splits(B, kvh, pages_per))
    ms = time_fn(lambda: model.forward(fb, kv), a.steps, warmup=2, graph=not a.eager)
    wbytes = w.nbytes()
    kvbytes = 2 * B * (a.ctx + 1) * cfg.num_layers * kvh * cfg.head_dim * 2
    pk = _peaks()
    return {"mode": "decode_step_eager" if a.eager else "decode_step_graph", "model": cfg.name, "tp": a.tp, "batch": B, "ctx": a.ctx, "ms": ms,
            "weight_bytes": wbytes, "kv_bytes": kvbytes,
            "roofline_ms": (wbytes + kvbytes) / pk["hbm_gbs"] / 1e6,
            "frac_of_roofline": (wbytes + kvbytes) / pk["hbm_gbs"] / 1e6 / ms}


def op_prefill_gemms(a):
    """The projection GEMMs of one batch prefill of the 8B shape (``--n`` tokens: QKV, o_proj,
    gate/up with the SwiGLU epilogue, down), ``--layers`` layers back to back, with the
    repo's tcgen05 GEMMs and with cuBLAS (``torch.matmul``, SwiGLU as separate ops), each
    sequence timed with CUDA events while the SM clock and throttle reasons are sampled: a
    seconds-long dense phase is where the 1 kW power cap sets the clock."""
    from ..ops import gemm
    from .timing import ClockSampler
    T, H, I, QKV = a.n, 4096, 14336, 6144
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(T, H, device="cuda", generator=g).bfloat16()
    W = {"qkv": (QKV, H), "o": (H, H), "gu": (2 * I, H), "d": (H, I)}
    W = {k: (torch.randn(*v, device="cuda", generator=g) * 0.02).bfloat16() for k, v in W.items()}
    flops = 2 * T * sum(w.shape[0] * w.shape[1] for w in W.values()) * a.layers

    def ours():
        for _ in range(a.layers):
            gemm.linear(x, W["qkv"])
            gemm.linear(x, W["o"])
            act = gemm.linear(x, W["gu"], swiglu=True)
            gemm.linear(act, W["d"])

    def cublas():
        for _ in range(a.layers):
            torch.matmul(x, W["qkv"].t())
            torch.matmul(x, W["o"].t())
            gu = torch.matmul(x, W["gu"].t())
            act = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
            torch.matmul(act, W["d"].t())

    out = {"op": "prefill_gemms", "tokens": T, "layers": a.layers, "TFLOP": flops / 1e12}
    for name, fn in (("ours", ours), ("cublas", cublas), ("ours_again", ours)):
        fn()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(torch.cuda.current_device(), period_ms=100) as clk:
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize()
        ms = s.elapsed_time(e)
        out[name] = {"ms": ms, "TFLOPs": flops / ms / 1e9, "clocks": clk.summary()}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", choices=["step", "gemm", "decode_attn", "prefill_attn", "mla_decode",
                                     "fp8_grouped", "gemm_ar1", "launch_floor", "prefill_gemms"],
                    default="step")
    ap.add_argument("--groups", type=int, default=48)
    ap.add_argument("--hq", type=int, default=32, help="decode_attn: query heads")
    ap.add_argument("--hkv", type=int, default=8, help="decode_attn: KV heads")
    ap.add_argument("--tp", type=int, default=1, help="step: time one rank of a TP group, no all-reduce")
    ap.add_argument("--model", default="llama-3-8b-shape")
    ap.add_argument("--layers", type=int, default=0)
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--m", type=int, default=4096)
    ap.add_argument("--n", type=int, default=32)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--swiglu", action="store_true")
    ap.add_argument("--splits", type=int, default=0, help="force K splits (0 = heuristic)")
    ap.add_argument("--eager", action="store_true", help="time eager launches (includes host overhead)")
    ap.add_argument("--kernel", default="tc", help="prefill_attn: tc (tcgen05) or mma (mma.sync)")
    a = ap.parse_args()
    out = {"step": decode_steps, "gemm": op_gemm, "decode_attn": op_decode_attn,
           "prefill_attn": op_prefill_attn,
           "mla_decode": op_mla_decode, "fp8_grouped": op_fp8_grouped,
           "gemm_ar1": op_gemm_ar1, "launch_floor": op_launch_floor,
           "prefill_gemms": op_prefill_gemms}[a.op](a)
    print(json.dumps(out))


if __name__ == "__main__":
    main()
