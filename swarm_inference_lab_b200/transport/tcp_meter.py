"""Byte-transparent TCP metering proxy (optionally TLS-terminating on the listen side).

Listens on a local port and forwards every accepted connection to an upstream
``host:port``, copying bytes in both directions unchanged while counting them per
connection and in total.  Used to account traffic of engines whose wire protocol
the runtime does not parse (e.g. an external RPC backend) and by the network
probes.

Reference: si/transport/tcp_meter.py:38.
"""
from __future__ import annotations

import asyncio
import ssl as _ssl
from dataclasses import dataclass, field


@dataclass
class MeterStats:
    connections: int = 0
    bytes_up: int = 0     # client -> upstream
    bytes_down: int = 0   # upstream -> client
    per_connection: list = field(default_factory=list)


class TcpMeterProxy:
    def __init__(self, upstream_host: str, upstream_port: int, *, host: str = "127.0.0.1",
                 port: int = 0, ssl_context: _ssl.SSLContext | None = None, chunk: int = 1 << 16):
        self.up = (upstream_host, upstream_port)
        self.host, self.port = host, port
        self.ssl = ssl_context
        self.chunk = chunk
        self.stats = MeterStats()
        self._server = None
        self._tasks: set[asyncio.Task] = set()

    async def start(self) -> int:
        self._server = await asyncio.start_server(self._handle, self.host, self.port, ssl=self.ssl)
        self.port = self._server.sockets[0].getsockname()[1]
        return self.port

    async def _pipe(self, reader, writer, rec: dict, key: str):
        try:
            while True:
                b = await reader.read(self.chunk)
                if not b:
                    break
                writer.write(b)
                await writer.drain()
                rec[key] += len(b)
                if key == "up":
                    self.stats.bytes_up += len(b)
                else:
                    self.stats.bytes_down += len(b)
        except (ConnectionError, asyncio.CancelledError):
            pass
        finally:
            try:
                writer.close()
            except Exception:  # noqa: BLE001
                pass

    async def _handle(self, creader, cwriter):
        self.stats.connections += 1
        rec = {"up": 0, "down": 0}
        self.stats.per_connection.append(rec)
        try:
            ureader, uwriter = await asyncio.open_connection(*self.up)
        except OSError:
            cwriter.close()
            return
        t1 = asyncio.create_task(self._pipe(creader, uwriter, rec, "up"))
        t2 = asyncio.create_task(self._pipe(ureader, cwriter, rec, "down"))
        self._tasks.update((t1, t2))
        await asyncio.gather(t1, t2, return_exceptions=True)
        self._tasks.difference_update((t1, t2))

    async def close(self):
        if self._server is not None:
            self._server.close()
            await self._server.wait_closed()
        for t in list(self._tasks):
            t.cancel()
