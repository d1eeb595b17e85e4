"""Per-device scratch owned by the kernel library.

Split-K GEMMs and split-KV decode attention write fp32 partials to a
workspace and count finished splits per output tile in an int32 counter
array; the last CTA of a tile reduces and re-arms its counter, so the
counters stay zero between launches.  The status word is the sticky device
error flag set by bounded waits inside the kernels (see ``csrc/include/sil/ptx.cuh``).

Kernels that share a workspace must run in stream order; a second stream
that runs kernels concurrently gets its own :class:`Workspace`.
"""
from __future__ import annotations

import threading

import torch

STATUS_NAMES = {
    0: "ok",
    1: "timeout waiting for a TMA stage",
    2: "timeout waiting for a free pipeline stage",
    3: "timeout waiting for the TMEM accumulator",
    4: "timeout waiting for a peer flag",
    5: "bad device-side argument",
    6: "timeout",
}


class KernelStatusError(RuntimeError):
    """A kernel's bounded wait gave up; the host turns the code into this error."""


class Workspace:
    def __init__(self, device: torch.device, fp32_elems: int = 16 << 20, counters: int = 1 << 16):
        self.device = torch.device(device)
        self.ws = torch.empty(fp32_elems, dtype=torch.float32, device=self.device)
        self.attn_ws = torch.empty(fp32_elems, dtype=torch.float32, device=self.device)
        self.counters = torch.zeros(counters, dtype=torch.int32, device=self.device)
        self.attn_counters = torch.zeros(counters, dtype=torch.int32, device=self.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)

    def check(self) -> None:
        """Raise :class:`KernelStatusError` if any kernel recorded a failure (syncs)."""
        code = int(self.status.item())
        if code != 0:
            raise KernelStatusError(f"device status {code}: {STATUS_NAMES.get(code, 'unknown')}")

    def reset(self) -> None:
        self.status.zero_()
        self.counters.zero_()
        self.attn_counters.zero_()


_local = threading.local()
_by_device: dict[tuple[str, int], Workspace] = {}
_lock = threading.Lock()


def get_workspace(device: torch.device | None = None) -> Workspace:
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if dev.index is None:
        dev = torch.device(dev.type, torch.cuda.current_device())
    key = (dev.type, dev.index)
    ws = _by_device.get(key)
    if ws is None:
        with _lock:
            ws = _by_device.get(key)
            if ws is None:
                ws = Workspace(dev)
                _by_device[key] = ws
    return ws
