"""Environment doctor: checks the pieces a stage owner needs on this machine.

Reads (never changes) GPU state through ``nvidia-smi`` queries and the CUDA
runtime, and reports whether the sm_100a kernel library and the native host
library are built and importable.  Reference: si/doctor.py:74-260.
"""
from __future__ import annotations

import shutil
import subprocess


def run_doctor() -> dict:
    rep: dict = {"checks": {}}
    c = rep["checks"]
    try:
        import torch
        c["torch"] = torch.__version__
        c["cuda_available"] = torch.cuda.is_available()
        if torch.cuda.is_available():
            p = torch.cuda.get_device_properties(0)
            c["gpu"] = p.name
            c["compute_capability"] = f"{p.major}.{p.minor}"
            c["sm_100a"] = (p.major, p.minor) == (10, 0)
    except Exception as exc:  # noqa: BLE001
        c["torch_error"] = str(exc)
    try:
        import importlib
        importlib.import_module("swarm_inference_lab_b200._C")
        c["kernel_library"] = "built"
    except Exception as exc:  # noqa: BLE001
        c["kernel_library"] = f"missing ({exc})"
    try:
        import importlib
        importlib.import_module("swarm_inference_lab_b200._native")
        c["native_library"] = "built"
    except Exception as exc:  # noqa: BLE001
        c["native_library"] = f"missing ({exc})"
    if shutil.which("nvidia-smi"):
        try:
            out = subprocess.run(["nvidia-smi", "--query-gpu=name,driver_version,memory.total",
                                  "--format=csv,noheader"], capture_output=True, text=True, timeout=10)
            c["nvidia_smi"] = out.stdout.strip().splitlines()
        except Exception as exc:  # noqa: BLE001
            c["nvidia_smi"] = f"error: {exc}"
    rep["ok"] = c.get("kernel_library") == "built" and (not c.get("cuda_available") or c.get("sm_100a", False))
    return rep
