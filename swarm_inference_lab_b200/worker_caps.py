"""Worker capability discovery and the planner-facing micro-benchmark.

``local_capabilities`` reports devices (name, SM count, memory, compute
capability), host memory and CPU count; with ``benchmark=True`` it also
measures what the planner needs on this node: HBM copy bandwidth and a
decode-shaped GEMM (the tcgen05 kernel at 32 tokens x 4096 x 4096) with
CUDA events.

Reference: si/worker/capabilities.py:57-568 (device/dtype/memory discovery,
decode-shaped matmul + copy benchmark).
"""
from __future__ import annotations

import os
import platform


def _host_memory_gb() -> float:
    try:
        import psutil
        return psutil.virtual_memory().total / 1e9
    except Exception:  # noqa: BLE001
        return 0.0


def local_capabilities(benchmark: bool = False) -> dict:
    caps = {"host": platform.node(), "os": platform.system(), "cpus": os.cpu_count(),
            "host_memory_gb": round(_host_memory_gb(), 1), "gpus": 0, "devices": []}
    try:
        import torch
        if torch.cuda.is_available():
            caps["gpus"] = torch.cuda.device_count()
            for i in range(caps["gpus"]):
                p = torch.cuda.get_device_properties(i)
                caps["devices"].append({"index": i, "name": p.name, "sm_count": p.multi_processor_count,
                                        "memory_gb": round(p.total_memory / 1e9, 1),
                                        "capability": f"{p.major}.{p.minor}"})
            caps["gpu_name"] = caps["devices"][0]["name"]
            if benchmark:
                caps["benchmark"] = measure_device_benchmark(0)
    except Exception as exc:  # noqa: BLE001
        caps["gpu_error"] = str(exc)
    return caps


def measure_device_benchmark(device: int = 0) -> dict:
    import torch
    from .utils.profile_decode import time_fn
    torch.cuda.set_device(device)
    a = torch.empty(1 << 30, dtype=torch.uint8, device="cuda")
    b = torch.empty_like(a)
    ms = time_fn(lambda: b.copy_(a), iters=10)
    out = {"copy_gbs": 2 * (1 << 30) / (ms / 1e3) / 1e9}
    del a, b
    try:
        from .ops import gemm
        x = torch.randn(32, 4096, device="cuda").bfloat16()
        w = torch.randn(4096, 4096, device="cuda").bfloat16()
        ms = time_fn(lambda: gemm.linear(x, w), iters=20)
        out["decode_gemm_us"] = ms * 1e3
        out["decode_gemm_gbs"] = w.numel() * 2 / (ms / 1e3) / 1e9
    except Exception as exc:  # noqa: BLE001
        out["decode_gemm_error"] = str(exc)
    return out
