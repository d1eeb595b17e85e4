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

from ..transport.stage_ring_net import TransportError

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

    def __init__(self, code: int):
        super().__init__(f"device status {code}: {STATUS_NAMES.get(code, 'unknown')}")
        self.code = code


class PeerTimeoutError(KernelStatusError, TransportError):
    """A peer GPU's flag never arrived within the wait limit (a transport failure of the
    NVLink data plane): the group must be rebuilt before its next collective."""


def error_for_status(code: int) -> KernelStatusError:
    """The host-side exception for a non-zero device status code."""
    return PeerTimeoutError(code) if code == 4 else KernelStatusError(code)


class Workspace:
    def __init__(self, device: torch.device, fp32_elems: int = 16 << 20, counters: int = 1 << 16):
        self.device = torch.device(device)
        self.ws = torch.empty(fp32_elems, dtype=torch.float32, device=self.device)
        self.attn_ws = torch.empty(fp32_elems, dtype=torch.float32, device=self.device)
        self.counters = torch.zeros(counters, dtype=torch.int32, device=self.device)
        self.attn_counters = torch.zeros(counters, dtype=torch.int32, device=self.device)
        # Status block: [0] sticky code, [1] unused, [2..3] wait limit in ns (uint64, 0 =
        # the kernels' compile-time default of 2 s).
        self.status = torch.zeros(4, dtype=torch.int32, device=self.device)

    def code(self) -> int:
        """The sticky status code (syncs)."""
        return int(self.status[0].item())

    def check(self) -> None:
        """Raise :class:`KernelStatusError` if any kernel recorded a failure (syncs)."""
        code = self.code()
        if code != 0:
            raise error_for_status(code)

    def set_wait_limit_ns(self, ns: int) -> None:
        """Bound every spin-wait of later launches to ``ns`` nanoseconds (0 = default 2 s).

        Stream-ordered on the current stream, so it applies to kernels launched after it.
        """
        self.status.view(torch.int64)[1].fill_(int(ns))

    def clear_status(self) -> None:
        """Clear the sticky code (keeps the wait limit)."""
        self.status[0].zero_()

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
