"""Topology domains for measured links.

A directed link is classified from its measured RTT, bandwidth, jitter and
stability.  ``NVLINK`` is the intra-box GPU-to-GPU domain (NVLink 5 /
NVSwitch, measured by ``parallel.nvlink_probe``); the others follow the
reference's host-network thresholds.

Reference: si/engines/topology.py:12-83 (LOCAL_FAST: RTT <= 5 ms,
BW >= 125 MB/s, jitter <= 2 ms, stability >= 0.98; REGIONAL: RTT <= 40 ms,
BW >= 12.5 MB/s; WAN; UNKNOWN).
"""
from __future__ import annotations

import enum
from dataclasses import dataclass


class Domain(str, enum.Enum):
    NVLINK = "nvlink"
    LOCAL_FAST = "local_fast"
    REGIONAL = "regional"
    WAN = "wan"
    UNKNOWN = "unknown"


@dataclass(frozen=True)
class LinkProfile:
    src: str
    dst: str
    rtt_ms: float | None
    bandwidth_MBps: float | None
    jitter_ms: float = 0.0
    stability: float = 1.0
    measured: bool = True
    kind: str = "tcp"          # tcp | nvlink
    latency_us: float | None = None  # one-way, NVLink probe


def classify(link: LinkProfile) -> Domain:
    if link.kind == "nvlink" and link.bandwidth_MBps:
        return Domain.NVLINK
    if link.rtt_ms is None or link.bandwidth_MBps is None or not link.measured:
        return Domain.UNKNOWN
    if (link.rtt_ms <= 5.0 and link.bandwidth_MBps >= 125.0 and link.jitter_ms <= 2.0
            and link.stability >= 0.98):
        return Domain.LOCAL_FAST
    if link.rtt_ms <= 40.0 and link.bandwidth_MBps >= 12.5:
        return Domain.REGIONAL
    return Domain.WAN


def transfer_ms(link: LinkProfile, nbytes: int) -> float:
    """One-way time for a message of ``nbytes`` on the link (latency + size / bandwidth)."""
    if link.kind == "nvlink":
        lat = (link.latency_us or 5.0) / 1000.0
    else:
        lat = (link.rtt_ms or 100.0) / 2.0
    bw = link.bandwidth_MBps or 1.0
    return lat + nbytes / (bw * 1e6) * 1e3
