"""Expert worker service: whole experts or microshards served over SWARMEX1.

A worker owns, per layer, a set of experts -- whole (all of the intermediate
dimension) or as microshards (a matched slice ``[i0, i1)`` of the gate, up and
down projections along the intermediate dimension).  A request carries token
rows, their routing (expert ids and weights, one entry per row and slot) and a
route-lease hash; the worker checks the hash against the leases it accepted,
computes SwiGLU per expert on the rows routed to it (``per_expert_exact``: one
output per (row, slot); ``per_worker_fast``: the weighted sum per row), and
replies.  Microshard partial outputs of one expert add up to the full expert
output; the caller reduces them in a fixed shard order in fp32
(``reduce_fixed_order``), so the result does not depend on arrival order.

Requests are admitted through a bounded queue (``max_inflight``); identical
requests (same request id and payload digest) are answered from a small LRU cache
(retries after a lost reply do not recompute).

Inside one B200 box experts are served by the fused expert-parallel path; this
service is the cross-host offload path.

Reference: si/worker/expert_service.py:95,352,390,558 (service, auth, queue, cache),
si/execution/microshard.py:15-162 (slice ownership, deterministic reconstruction).
"""
from __future__ import annotations

import asyncio
import hashlib
from collections import OrderedDict
from dataclasses import dataclass

import torch

from ..transport.expert_wire import ExpertPacket, decode_tensor, encode_tensor, read_packet, write_packet


@dataclass(frozen=True)
class Microshard:
    layer: int
    expert: int
    i0: int
    i1: int           # intermediate slice [i0, i1)

    def covers_whole(self, inter: int) -> bool:
        return self.i0 == 0 and self.i1 == inter


def split_microshards(layer: int, expert: int, inter: int, parts: int) -> list[Microshard]:
    """Matched contiguous slices of the intermediate dimension (equal up to one row)."""
    base, rem = divmod(inter, parts)
    out, s = [], 0
    for i in range(parts):
        n = base + (1 if i < rem else 0)
        out.append(Microshard(layer, expert, s, s + n))
        s += n
    return out


def reduce_fixed_order(partials: dict[int, torch.Tensor]) -> torch.Tensor:
    """Sum microshard partial outputs in shard-index order, in fp32."""
    acc = None
    for k in sorted(partials):
        acc = partials[k].float() if acc is None else acc + partials[k].float()
    return acc


class ExpertStore:
    """Expert weights held by one worker: w_gate/w_up [I, H], w_down [H, I] per (layer, expert),
    restricted to the owned slice."""

    def __init__(self, device="cpu", dtype=torch.float32):
        self.device = torch.device(device)
        self.dtype = dtype
        self.w: dict[tuple[int, int], tuple[Microshard, torch.Tensor, torch.Tensor, torch.Tensor]] = {}

    def add(self, shard: Microshard, gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor) -> None:
        g = gate[shard.i0:shard.i1].to(self.device, self.dtype)
        u = up[shard.i0:shard.i1].to(self.device, self.dtype)
        d = down[:, shard.i0:shard.i1].to(self.device, self.dtype)
        self.w[(shard.layer, shard.expert)] = (shard, g, u, d)

    def owns(self, layer: int, expert: int) -> bool:
        return (layer, expert) in self.w

    def forward(self, layer: int, expert: int, x: torch.Tensor) -> torch.Tensor:
        _, g, u, d = self.w[(layer, expert)]
        x = x.to(self.device, self.dtype)
        return (torch.nn.functional.silu(x @ g.T) * (x @ u.T)) @ d.T


class ExpertService:
    def __init__(self, store: ExpertStore, *, host: str = "127.0.0.1", port: int = 0,
                 max_inflight: int = 8, cache_entries: int = 64):
        self.store = store
        self.host, self.port = host, port
        self.accepted_leases: set[str] = set()
        self._sem = asyncio.Semaphore(max_inflight)
        self._cache: OrderedDict[str, ExpertPacket] = OrderedDict()
        self._cache_n = cache_entries
        self.stats = {"requests": 0, "rejected": 0, "cache_hits": 0, "rows": 0}
        self._server = None
        self._writers: set = set()

    def accept_lease(self, lease_hash: str) -> None:
        self.accepted_leases.add(lease_hash)

    async def start(self) -> int:
        self._server = await asyncio.start_server(self._conn, self.host, self.port)
        self.port = self._server.sockets[0].getsockname()[1]
        return self.port

    async def close(self):
        if self._server is not None:
            self._server.close()
            for w in list(self._writers):
                w.close()
            await self._server.wait_closed()

    async def _conn(self, reader, writer):
        self._writers.add(writer)
        try:
            while True:
                req = await read_packet(reader, timeout=None)
                async with self._sem:
                    rep = self.handle(req)
                await write_packet(writer, rep)
        except (asyncio.IncompleteReadError, ConnectionError):
            pass
        finally:
            self._writers.discard(writer)
            writer.close()

    def _error(self, req: ExpertPacket, msg: str) -> ExpertPacket:
        return ExpertPacket({"kind": "expert_response", "status": "ERROR", "error": msg,
                             "request_id": req.header.get("request_id")})

    def handle(self, req: ExpertPacket) -> ExpertPacket:
        h = req.header
        self.stats["requests"] += 1
        if h.get("kind") != "expert_request":
            return self._error(req, "not an expert request")
        if h.get("route_lease_hash") not in self.accepted_leases:
            self.stats["rejected"] += 1
            return self._error(req, "route lease not accepted")
        key = h.get("request_id", "") + ":" + hashlib.sha256(b"".join(req.blobs)).hexdigest()
        if key in self._cache:
            self.stats["cache_hits"] += 1
            self._cache.move_to_end(key)
            return self._cache[key]
        layer = int(h["layer"])
        x = decode_tensor(req, "rows")                       # [R, H]
        ids = decode_tensor(req, "expert_ids").long()        # [R, k]
        wts = decode_tensor(req, "weights")                  # [R, k]
        mode = h.get("response_mode", "per_worker_fast")
        R, K = ids.shape
        per = torch.zeros(R, K, x.shape[1])
        owned = torch.zeros(R, K, dtype=torch.bool)
        for e in torch.unique(ids).tolist():
            if not self.store.owns(layer, e):
                continue
            m = ids == e
            r_idx, s_idx = m.nonzero(as_tuple=True)
            y = self.store.forward(layer, e, x[r_idx]).float().cpu()
            per[r_idx, s_idx] = y
            owned[r_idx, s_idx] = True
        self.stats["rows"] += R
        rep = ExpertPacket({"kind": "expert_response", "status": "OK", "request_id": h.get("request_id"),
                            "layer": layer, "response_mode": mode})
        codec = h.get("codec", "raw_fp32")
        if mode == "per_expert_exact":
            encode_tensor(rep, "outputs", per, codec)
            encode_tensor(rep, "owned", owned.float(), "raw_fp32")
        else:
            encode_tensor(rep, "weighted_sum", (per * wts[..., None]).sum(1), codec)
        self._cache[key] = rep
        while len(self._cache) > self._cache_n:
            self._cache.popitem(last=False)
        return rep


class ExpertClient:
    def __init__(self, host: str, port: int, *, timeout: float = 30.0):
        self.host, self.port, self.timeout = host, port, timeout
        self._rw = None

    async def _conn(self):
        if self._rw is None:
            self._rw = await asyncio.wait_for(asyncio.open_connection(self.host, self.port), self.timeout)
        return self._rw

    async def run(self, *, request_id: str, layer: int, rows: torch.Tensor, expert_ids: torch.Tensor,
                  weights: torch.Tensor, lease_hash: str, mode: str = "per_worker_fast",
                  codec: str = "raw_fp32") -> ExpertPacket:
        p = ExpertPacket({"kind": "expert_request", "request_id": request_id, "layer": layer,
                          "route_lease_hash": lease_hash, "response_mode": mode, "codec": codec})
        encode_tensor(p, "rows", rows, codec)
        encode_tensor(p, "expert_ids", expert_ids.float(), "raw_fp32")
        encode_tensor(p, "weights", weights, "raw_fp32")
        reader, writer = await self._conn()
        await write_packet(writer, p)
        return await read_packet(reader, self.timeout)

    def close(self):
        if self._rw is not None:
            self._rw[1].close()
            self._rw = None
