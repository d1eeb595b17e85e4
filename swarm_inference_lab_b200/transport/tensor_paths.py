"""Tensor paths between stage owners, chosen by locality.

* ``InProcessPath``: producer and consumer share a process and device -- hand over
  the tensor itself (no copy), ordered by a CUDA event on the producer's stream.
* ``PinnedStagingPath``: different processes on one host without peer access --
  asynchronous device -> pinned host copy on a side stream, the consumer copies
  pinned -> device; the event keeps the two in order.
* ``FramePath``: remote peers -- little-endian bytes with dtype and shape (the
  stage-ring payload; ``tensor_codec``).

Inside a B200 box stage boundaries use NCCL p2p (``parallel/pipeline.py``);
these paths serve loopback, host-staged and cross-host links.

Reference: si/transport/tensor_paths.py:17-244.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .tensor_codec import pack_tensor, unpack_tensor


@dataclass
class Handoff:
    tensor: torch.Tensor | None = None
    event: object = None
    frame: bytes | None = None
    meta: dict | None = None


class InProcessPath:
    name = "in_process"

    def send(self, t: torch.Tensor) -> Handoff:
        ev = None
        if t.is_cuda:
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(t.device))
        return Handoff(tensor=t, event=ev)

    def recv(self, h: Handoff, device=None) -> torch.Tensor:
        if h.event is not None:
            torch.cuda.current_stream(h.tensor.device).wait_event(h.event)
        return h.tensor if device is None else h.tensor.to(device, non_blocking=True)


class PinnedStagingPath:
    name = "pinned_staging"

    def __init__(self):
        self._bufs: dict[tuple, torch.Tensor] = {}

    def _buf(self, t: torch.Tensor) -> torch.Tensor:
        key = (tuple(t.shape), t.dtype)
        b = self._bufs.get(key)
        if b is None:
            b = torch.empty(t.shape, dtype=t.dtype, pin_memory=torch.cuda.is_available())
            self._bufs[key] = b
        return b

    def send(self, t: torch.Tensor) -> Handoff:
        b = self._buf(t)
        if t.is_cuda:
            s = torch.cuda.Stream(t.device)
            s.wait_stream(torch.cuda.current_stream(t.device))
            with torch.cuda.stream(s):
                b.copy_(t, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(s)
            return Handoff(tensor=b, event=ev)
        b.copy_(t)
        return Handoff(tensor=b)

    def recv(self, h: Handoff, device=None) -> torch.Tensor:
        if h.event is not None:
            h.event.synchronize()
        return h.tensor.to(device, non_blocking=True) if device is not None else h.tensor.clone()


class FramePath:
    name = "frame"

    def send(self, t: torch.Tensor) -> Handoff:
        p = pack_tensor(t)
        return Handoff(frame=p.payload, meta=p.attributes)

    def recv(self, h: Handoff, device=None) -> torch.Tensor:
        t = unpack_tensor(h.frame, h.meta)
        return t.to(device) if device is not None else t


def choose_path(same_process: bool, same_host: bool, peer_access: bool):
    if same_process:
        return InProcessPath()
    if same_host and not peer_access:
        return PinnedStagingPath()
    return FramePath()
