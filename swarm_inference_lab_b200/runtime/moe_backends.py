"""MoE execution backends for a stage: where each routed expert of a layer runs.

A backend computes, for token rows ``x`` [R, H] with routing ``ids`` / ``weights`` [R, k],
the weighted sum over the k slots of the experts' SwiGLU outputs ([R, H], fp32):

* ``LocalMoEBackend``            every expert in this process (an ``ExpertStore``);
* ``WholeExpertRemoteBackend``   each expert on one remote expert worker (SWARMEX1), one
                                 request per worker per layer, per-(row, slot) outputs back;
* ``MicroshardRemoteBackend``    each expert's intermediate dimension split across several
                                 workers; the partial outputs are added in shard order (fp32)
                                 before the weighting, so arrival order never matters;
* ``HybridMoEBackend``           per (layer, expert) one of the above, from the expert
                                 planner's decisions (``planner/expert_planner.py``).

All backends combine slots in the same order (slot 0..k-1 per row), so switching a
placement changes results only at fp32 rounding.  Backends are synchronous for the stage
executor (which runs in a worker thread); network calls run on a private event loop.

Reference: si/execution/moe.py:433-1555 (``LocalMoeBackend``, ``WholeExpertRemoteBackend``,
``MicroshardRemoteBackend``, ``HybridMoeBackend``).
"""
from __future__ import annotations

import asyncio
import itertools
import threading

import torch

from .expert_service import ExpertClient, ExpertStore, reduce_fixed_order


class _Loop:
    """A private asyncio loop in a daemon thread, for synchronous callers."""

    def __init__(self):
        self.loop = asyncio.new_event_loop()
        self.thread = threading.Thread(target=self.loop.run_forever, daemon=True)
        self.thread.start()

    def run(self, coro, timeout: float = 120.0):
        return asyncio.run_coroutine_threadsafe(coro, self.loop).result(timeout)

    def close(self):
        self.loop.call_soon_threadsafe(self.loop.stop)
        self.thread.join(timeout=5)


def combine_slots(per: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
    """sum_k weights[r, k] * per[r, k, :] in slot order (fp32)."""
    out = torch.zeros(per.shape[0], per.shape[2], dtype=torch.float32)
    for k in range(per.shape[1]):
        out += weights[:, k:k + 1].float() * per[:, k].float()
    return out


class LocalMoEBackend:
    kind = "local"

    def __init__(self, store: ExpertStore):
        self.store = store

    def per_slot(self, layer: int, x: torch.Tensor, ids: torch.Tensor, mask: torch.Tensor | None = None
                 ) -> torch.Tensor:
        R, K = ids.shape
        per = torch.zeros(R, K, x.shape[1], dtype=torch.float32)
        for e in torch.unique(ids).tolist():
            sel = ids == e
            if mask is not None:
                sel = sel & mask
            if not sel.any():
                continue
            r, s = sel.nonzero(as_tuple=True)
            per[r, s] = self.store.forward(layer, e, x[r]).float().cpu()
        return per

    def experts(self, layer: int, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
        return combine_slots(self.per_slot(layer, x, ids), weights)


class _RemoteBase:
    def __init__(self, lease_hash: str):
        self.lease_hash = lease_hash
        self._loop = _Loop()
        self._ids = itertools.count()
        self.requests = 0

    async def _ask(self, client: ExpertClient, layer: int, x, ids, weights):
        rep = await client.run(request_id=f"moe-{next(self._ids)}", layer=layer, rows=x,
                               expert_ids=ids, weights=weights, lease_hash=self.lease_hash,
                               mode="per_expert_exact")
        if rep.header.get("status") != "OK":
            raise RuntimeError(f"expert worker: {rep.header.get('error')}")
        from ..transport.expert_wire import decode_tensor
        self.requests += 1
        return decode_tensor(rep, "outputs").float(), decode_tensor(rep, "owned").bool()

    def clients(self):
        return []

    def close(self):
        async def shut():
            for c in self.clients():
                c.close()
        self._loop.run(shut())
        self._loop.close()


class WholeExpertRemoteBackend(_RemoteBase):
    """``owner[(layer, expert)] -> ExpertClient`` of the worker holding the whole expert."""
    kind = "whole_remote"

    def __init__(self, owner: dict, lease_hash: str):
        super().__init__(lease_hash)
        self.owner = owner

    def clients(self):
        return list({id(c): c for c in self.owner.values()}.values())

    def per_slot(self, layer: int, x, ids, mask=None) -> torch.Tensor:
        R, K = ids.shape
        per = torch.zeros(R, K, x.shape[1], dtype=torch.float32)
        clients = {}
        for e in torch.unique(ids).tolist():
            c = self.owner.get((layer, e))
            if c is not None and (mask is None or ((ids == e) & mask).any()):
                clients[id(c)] = c
        if not clients:
            return per

        sent = ids if mask is None else torch.where(mask, ids, torch.full_like(ids, -1))

        async def gather():
            return await asyncio.gather(*[self._ask(c, layer, x, sent, torch.ones_like(ids, dtype=torch.float32))
                                          for c in clients.values()])
        for out, owned in self._loop.run(gather()):
            sel = owned if mask is None else owned & mask
            per[sel] = out[sel]
        return per

    def experts(self, layer, x, ids, weights):
        return combine_slots(self.per_slot(layer, x, ids), weights)


class MicroshardRemoteBackend(_RemoteBase):
    """``shards[(layer, expert)] -> [ExpertClient, ...]`` in shard order; each holds one
    slice of the intermediate dimension."""
    kind = "microshard"

    def __init__(self, shards: dict, lease_hash: str):
        super().__init__(lease_hash)
        self.shards = shards

    def clients(self):
        return list({id(c): c for cl in self.shards.values() for c in cl}.values())

    def per_slot(self, layer: int, x, ids, mask=None) -> torch.Tensor:
        R, K = ids.shape
        per = torch.zeros(R, K, x.shape[1], dtype=torch.float32)
        experts = [e for e in torch.unique(ids).tolist() if (layer, e) in self.shards
                   and (mask is None or ((ids == e) & mask).any())]
        for e in experts:
            sel = ids == e
            if mask is not None:
                sel = sel & mask
            clients = self.shards[(layer, e)]
            # Ask every shard for this expert only (other slots are marked with id -1).
            only = torch.where(sel, ids, torch.full_like(ids, -1))

            async def gather(cl=clients, only=only):
                return await asyncio.gather(*[self._ask(c, layer, x, only,
                                                        torch.ones_like(only, dtype=torch.float32))
                                              for c in cl])
            parts = self._loop.run(gather())
            full = reduce_fixed_order({i: out for i, (out, _) in enumerate(parts)})
            per[sel] = full[sel]
        return per

    def experts(self, layer, x, ids, weights):
        return combine_slots(self.per_slot(layer, x, ids), weights)


class HybridMoEBackend:
    """Per (layer, expert) placement: ``local``, ``whole_remote`` or ``microshard`` backends,
    chosen by ``placement[(layer, expert)]`` (the expert planner's decisions)."""
    kind = "hybrid"

    def __init__(self, placement: dict, *, local: LocalMoEBackend | None = None,
                 whole: WholeExpertRemoteBackend | None = None,
                 micro: MicroshardRemoteBackend | None = None):
        self.placement = placement
        self.backends = {"local": local, "whole_remote": whole, "microshard": micro}

    @classmethod
    def from_decisions(cls, decisions, **backends) -> "HybridMoEBackend":
        return cls({(d.layer, d.expert): ("microshard" if d.placement == "hybrid" else d.placement)
                    for d in decisions}, **backends)

    def experts(self, layer: int, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
        R, K = ids.shape
        per = torch.zeros(R, K, x.shape[1], dtype=torch.float32)
        kind = torch.empty_like(ids)
        names = ["local", "whole_remote", "microshard"]
        for e in torch.unique(ids).tolist():
            p = self.placement.get((layer, e), "local")
            kind[ids == e] = names.index(p)
        for i, name in enumerate(names):
            mask = kind == i
            if not mask.any():
                continue
            be = self.backends[name]
            if be is None:
                raise RuntimeError(f"no {name} backend for experts placed there")
            part = be.per_slot(layer, x, ids, mask)
            per[mask] = part[mask]
        return combine_slots(per, weights)
