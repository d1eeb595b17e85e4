"""Directed network measurement between workers, authorised by signed probe tickets.

The coordinator issues a ticket ``{src, dst, bytes, nonce, expires_at}`` signed with
its identity; the destination worker's ``ProbeServer`` accepts a probe only with a
valid, unexpired, unused ticket naming it.  A probe measures the directed link
src -> dst:

* RTT: ``pings`` one-byte round trips (p50, jitter = p90 - p10);
* upload: ``bytes`` sent src -> dst, timed until dst acknowledges the last byte;
* download: ``bytes`` sent dst -> src;
* stability: 1 - coefficient of variation of the RTT samples.

Results go to a ``LinkRepository`` keyed by (src, dst) with a TTL; the planner only
uses fresh measurements and falls back to its defaults for stale links.

Inside one B200 box NVLink is measured by ``parallel/nvlink_probe.py``; this module
covers the host network between boxes.

Reference: si/cluster/network.py:164 (server), :395 ``DirectedNetworkMeasurer``,
:460-604 measure, :620 freshness, :633 repository.
"""
from __future__ import annotations

import asyncio
import json
import secrets
import statistics
import time
from dataclasses import asdict, dataclass

from ..security.identity import Identity, SignatureError, sign_record, verify_record

CHUNK = 1 << 16


def issue_ticket(coordinator: Identity, src: str, dst: str, nbytes: int = 4 << 20,
                 ttl_s: float = 60.0) -> dict:
    return sign_record(coordinator, {"kind": "probe_ticket", "src": src, "dst": dst,
                                     "bytes": int(nbytes), "nonce": secrets.token_hex(12),
                                     "expires_at": time.time() + ttl_s})


@dataclass
class LinkMeasurement:
    src: str
    dst: str
    rtt_ms: float
    jitter_ms: float
    upload_Bps: float
    download_Bps: float
    stability: float
    measured_at: float

    def to_json(self) -> dict:
        return asdict(self)


class ProbeServer:
    def __init__(self, worker_id: str, coordinator_fingerprint: str, *, host: str = "127.0.0.1",
                 port: int = 0, max_bytes: int = 256 << 20):
        self.worker_id = worker_id
        self.trusted = {coordinator_fingerprint}
        self.host, self.port = host, port
        self.max_bytes = max_bytes
        self._nonces: set[str] = set()
        self._server = None
        self.rejected = 0

    async def start(self) -> int:
        self._server = await asyncio.start_server(self._handle, self.host, self.port)
        self.port = self._server.sockets[0].getsockname()[1]
        return self.port

    def _check(self, signed: dict) -> dict:
        body = verify_record(signed, self.trusted)
        if body.get("kind") != "probe_ticket" or body.get("dst") != self.worker_id:
            raise SignatureError("ticket not for this worker")
        if body["expires_at"] < time.time():
            raise SignatureError("ticket expired")
        if body["nonce"] in self._nonces:
            raise SignatureError("ticket replayed")
        if body["bytes"] > self.max_bytes:
            raise SignatureError("ticket asks for too many bytes")
        self._nonces.add(body["nonce"])
        return body

    async def _handle(self, reader, writer):
        try:
            line = await asyncio.wait_for(reader.readline(), 10)
            try:
                t = self._check(json.loads(line))
            except (SignatureError, ValueError, KeyError) as exc:
                self.rejected += 1
                writer.write(json.dumps({"ok": False, "error": str(exc)}).encode() + b"\n")
                await writer.drain()
                return
            writer.write(b'{"ok": true}\n')
            await writer.drain()
            # ping phase: echo single bytes until a zero byte
            while True:
                b = await reader.readexactly(1)
                writer.write(b)
                await writer.drain()
                if b == b"\0":
                    break
            # upload phase: read n bytes, ack
            n = t["bytes"]
            got = 0
            while got < n:
                chunk = await reader.read(min(CHUNK, n - got))
                if not chunk:
                    raise ConnectionError("probe client went away")
                got += len(chunk)
            writer.write(b"A")
            await writer.drain()
            # download phase
            buf = b"\x5a" * CHUNK
            sent = 0
            while sent < n:
                k = min(CHUNK, n - sent)
                writer.write(buf[:k])
                sent += k
            await writer.drain()
        except (asyncio.IncompleteReadError, ConnectionError, asyncio.TimeoutError):
            pass
        finally:
            writer.close()

    async def close(self):
        if self._server is not None:
            self._server.close()
            await self._server.wait_closed()


class DirectedNetworkMeasurer:
    def __init__(self, src: str, *, pings: int = 20, timeout_s: float = 30.0):
        self.src = src
        self.pings = pings
        self.timeout = timeout_s

    async def measure(self, host: str, port: int, ticket: dict) -> LinkMeasurement:
        reader, writer = await asyncio.wait_for(asyncio.open_connection(host, port), self.timeout)
        try:
            writer.write(json.dumps(ticket).encode() + b"\n")
            await writer.drain()
            resp = json.loads(await asyncio.wait_for(reader.readline(), self.timeout))
            if not resp.get("ok"):
                raise SignatureError(resp.get("error", "probe refused"))
            rtts = []
            for i in range(self.pings):
                t0 = time.perf_counter()
                writer.write(b"\1")
                await writer.drain()
                await asyncio.wait_for(reader.readexactly(1), self.timeout)
                rtts.append(time.perf_counter() - t0)
            writer.write(b"\0")
            await writer.drain()
            await reader.readexactly(1)
            n = int(ticket["bytes"])
            buf = b"\xa5" * CHUNK
            t0 = time.perf_counter()
            sent = 0
            while sent < n:
                k = min(CHUNK, n - sent)
                writer.write(buf[:k])
                sent += k
                if sent % (16 * CHUNK) == 0:
                    await writer.drain()
            await writer.drain()
            await asyncio.wait_for(reader.readexactly(1), self.timeout)
            up = n / max(time.perf_counter() - t0, 1e-9)
            t0 = time.perf_counter()
            got = 0
            while got < n:
                chunk = await asyncio.wait_for(reader.read(CHUNK), self.timeout)
                if not chunk:
                    break
                got += len(chunk)
            down = got / max(time.perf_counter() - t0, 1e-9)
        finally:
            writer.close()
        rs = sorted(rtts)
        p50 = statistics.median(rs)
        p10, p90 = rs[int(0.1 * (len(rs) - 1))], rs[int(0.9 * (len(rs) - 1))]
        mean = statistics.fmean(rs)
        cv = statistics.pstdev(rs) / mean if mean > 0 else 0.0
        return LinkMeasurement(self.src, ticket["dst"], p50 * 1e3, (p90 - p10) * 1e3, up, down,
                               max(0.0, 1.0 - cv), time.time())


class LinkRepository:
    """Latest measurement per directed link, with TTL freshness."""

    def __init__(self, ttl_s: float = 600.0):
        self.ttl = ttl_s
        self.links: dict[tuple[str, str], LinkMeasurement] = {}

    def record(self, m: LinkMeasurement) -> None:
        self.links[(m.src, m.dst)] = m

    def fresh(self, src: str, dst: str, *, now: float | None = None) -> LinkMeasurement | None:
        m = self.links.get((src, dst))
        now = time.time() if now is None else now
        if m is None or now - m.measured_at > self.ttl:
            return None
        return m

    def stale_links(self, pairs: list[tuple[str, str]], *, now: float | None = None) -> list[tuple[str, str]]:
        return [p for p in pairs if self.fresh(*p, now=now) is None]

    def to_json(self) -> list[dict]:
        return [m.to_json() for m in self.links.values()]
