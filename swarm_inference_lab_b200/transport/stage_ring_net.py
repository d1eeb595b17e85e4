"""Asyncio TCP (optionally TLS 1.3) transport for SWRING01 frames.

* ``read_frame`` / ``write_frame``: frame boundaries come only from the fixed
  header lengths; partial reads are handled by ``readexactly``.
* ``StageRingServer``: bounded number of connections; each connection is
  served in order by an async handler returning zero or more reply frames.
* ``StageRingConnection``: one ordered, pipelined connection to a peer
  (replies matched FIFO), with an optional fault injector consulted before
  every send.
* ``ConnectionPool``: one connection per peer, reconnect on demand, poisoned
  connections evicted after a transport error.

Transport errors (EOF, reset, integrity failure, timeout) surface as
:class:`TransportError`, which the coordinator turns into a recovery.

Reference behaviour: si/transport/stage_ring_connection.py:104-475,
si/transport/stage_ring_server.py:90, si/transport/stage_ring_faults.py:84-149.
"""
from __future__ import annotations

import asyncio
import ssl
from collections import deque
from dataclasses import dataclass, field
from typing import Awaitable, Callable

from ..protocol import stage_ring as sr


class TransportError(ConnectionError):
    pass


async def read_frame(reader: asyncio.StreamReader, timeout: float | None = None) -> sr.StageMessage:
    try:
        head = await asyncio.wait_for(reader.readexactly(sr.HEADER_SIZE), timeout)
        h = sr.decode_header(head)
        body = await asyncio.wait_for(reader.readexactly(h.body_length), timeout)
    except asyncio.IncompleteReadError as exc:
        raise TransportError("connection closed mid-frame" if exc.partial else "connection closed") from None
    except (ConnectionError, OSError) as exc:
        raise TransportError(str(exc)) from None
    except asyncio.TimeoutError:
        raise TransportError("receive timed out") from None
    try:
        return sr.decode_body(h, body)
    except sr.FrameError as exc:
        raise TransportError(f"integrity failure: {exc}") from None


async def write_frame(writer: asyncio.StreamWriter, msg: sr.StageMessage) -> int:
    data = sr.encode(msg)
    try:
        writer.write(data)
        await writer.drain()
    except (ConnectionError, OSError) as exc:
        raise TransportError(str(exc)) from None
    return len(data)


Handler = Callable[[sr.StageMessage], Awaitable[list[sr.StageMessage]]]


@dataclass
class ServerStats:
    connections: int = 0
    frames_in: int = 0
    frames_out: int = 0
    bytes_out: int = 0
    rejected: int = 0


class StageRingServer:
    def __init__(self, handler: Handler, host: str = "127.0.0.1", port: int = 0,
                 ssl_context: ssl.SSLContext | None = None, max_connections: int = 64,
                 idle_timeout: float | None = None):
        self.handler = handler
        self.host, self.port = host, port
        self.ssl = ssl_context
        self.max_connections = max_connections
        self.idle_timeout = idle_timeout
        self.stats = ServerStats()
        self._server: asyncio.base_events.Server | None = None
        self._conns: set[asyncio.StreamWriter] = set()

    async def start(self) -> int:
        self._server = await asyncio.start_server(self._serve, self.host, self.port, ssl=self.ssl)
        self.port = self._server.sockets[0].getsockname()[1]
        return self.port

    async def _serve(self, reader, writer):
        if len(self._conns) >= self.max_connections:
            self.stats.rejected += 1
            writer.close()
            return
        self._conns.add(writer)
        self.stats.connections += 1
        try:
            while True:
                try:
                    msg = await read_frame(reader, self.idle_timeout)
                except TransportError:
                    break
                self.stats.frames_in += 1
                replies = await self.handler(msg)
                for r in replies:
                    self.stats.bytes_out += await write_frame(writer, r)
                    self.stats.frames_out += 1
        except TransportError:
            pass
        finally:
            self._conns.discard(writer)
            writer.close()

    async def close(self) -> None:
        if self._server is not None:
            self._server.close()
            for w in list(self._conns):
                w.close()
            await self._server.wait_closed()
            self._server = None

    def drop_connections(self) -> None:
        """Close every live connection (fault drills)."""
        for w in list(self._conns):
            w.close()


class FaultInjector:
    """Consulted before each send; return True to make the send fail."""

    def before_send(self, conn: "StageRingConnection", msg: sr.StageMessage) -> bool:
        return False


@dataclass
class CloseBeforeSend(FaultInjector):
    """Close the active connection right before sending the n-th matching frame."""

    operation: sr.Operation = sr.Operation.DECODE
    token_position: int | None = None
    times: int = 1
    fired: int = 0
    seen: list = field(default_factory=list)

    def before_send(self, conn, msg):
        if self.fired >= self.times or msg.operation != self.operation:
            return False
        if self.token_position is not None and msg.token_position != self.token_position:
            return False
        self.fired += 1
        self.seen.append((msg.session_id, msg.token_position))
        conn.writer.close()
        return True


class StageRingConnection:
    def __init__(self, reader, writer, *, timeout: float = 30.0, fault: FaultInjector | None = None):
        self.reader, self.writer = reader, writer
        self.timeout = timeout
        self.fault = fault
        self._pending: deque[asyncio.Future] = deque()
        self._send_lock = asyncio.Lock()
        self._reader_task = asyncio.ensure_future(self._read_loop())
        self.closed = False
        self.bytes_sent = 0

    @classmethod
    async def open(cls, host: str, port: int, *, ssl_context=None, timeout: float = 30.0,
                   fault: FaultInjector | None = None, server_hostname: str | None = None):
        try:
            r, w = await asyncio.wait_for(
                asyncio.open_connection(host, port, ssl=ssl_context,
                                        server_hostname=server_hostname if ssl_context else None),
                timeout)
        except (OSError, asyncio.TimeoutError) as exc:
            raise TransportError(f"connect {host}:{port}: {exc}") from None
        return cls(r, w, timeout=timeout, fault=fault)

    async def _read_loop(self):
        try:
            while True:
                msg = await read_frame(self.reader)
                if not self._pending:
                    continue  # unsolicited frame: ignore
                fut = self._pending.popleft()
                if not fut.done():
                    fut.set_result(msg)
        except TransportError as exc:
            self._fail(exc)
        except asyncio.CancelledError:
            self._fail(TransportError("connection closed"))

    def _fail(self, exc: Exception):
        self.closed = True
        while self._pending:
            fut = self._pending.popleft()
            if not fut.done():
                fut.set_exception(TransportError(str(exc)))

    async def request(self, msg: sr.StageMessage, expect_reply: bool = True) -> sr.StageMessage | None:
        if self.closed:
            raise TransportError("connection is closed")
        fut = asyncio.get_running_loop().create_future() if expect_reply else None
        async with self._send_lock:
            if self.fault is not None and self.fault.before_send(self, msg):
                self.closed = True
                raise TransportError("connection closed by fault injector before send")
            if fut is not None:
                self._pending.append(fut)
            self.bytes_sent += await write_frame(self.writer, msg)
        if fut is None:
            return None
        try:
            return await asyncio.wait_for(fut, self.timeout)
        except asyncio.TimeoutError:
            self.close()
            raise TransportError("reply timed out") from None

    def close(self):
        self.closed = True
        self._reader_task.cancel()
        self.writer.close()


class ConnectionPool:
    """One connection per peer address; evicts a connection after a transport error."""

    def __init__(self, *, ssl_context=None, timeout: float = 30.0, fault: FaultInjector | None = None):
        self.ssl = ssl_context
        self.timeout = timeout
        self.fault = fault
        self._conns: dict[tuple[str, int], StageRingConnection] = {}
        self.reconnects = 0

    async def get(self, host: str, port: int) -> StageRingConnection:
        key = (host, port)
        c = self._conns.get(key)
        if c is None or c.closed:
            if c is not None:
                self.reconnects += 1
            c = await StageRingConnection.open(host, port, ssl_context=self.ssl,
                                               timeout=self.timeout, fault=self.fault)
            self._conns[key] = c
        return c

    async def send(self, host: str, port: int, msg: sr.StageMessage) -> sr.StageMessage:
        c = await self.get(host, port)
        try:
            return await c.request(msg)
        except TransportError:
            c.close()
            self._conns.pop((host, port), None)
            raise

    async def close(self):
        for c in self._conns.values():
            c.close()
        self._conns.clear()
