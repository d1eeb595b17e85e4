"""A fault-injecting TCP proxy in front of a SWRING01 endpoint (stage owner).

The proxy listens on its own port and forwards whole frames in both directions to the
target endpoint, so the real transport, codec and stage owner run unchanged on either
side.  Per proxy, faults can be switched on at any time:

* ``delay_s``          every forwarded request frame waits this long first (WAN latency);
* ``reply_delay_s``    the same for reply frames (one-way latency of the return path);
* ``disconnected``     new connections are closed at once and open ones are dropped;
* ``corrupt_next``     the next reply frame gets one payload (or metadata) bit flipped, so
                       the receiver's SHA-256 check rejects it (an integrity failure);
* ``timeout_next``     the next request frame is swallowed: no reply ever comes, and the
                       caller's receive deadline fires.

Forwarded traffic is counted per direction (frames and body bytes: ``stats``).  Every
injected fault is recorded in ``events`` (kind, time, frame operation), separate from
the measured transport, so a run can tell emulated faults from real ones.

Reference: si/transport/fault_proxy.py:26-107 (``EndpointFault``: delay, disconnect, corrupt
activation, timeout; observable events).
"""
from __future__ import annotations

import asyncio
import time
from dataclasses import dataclass, field

from ..protocol import stage_ring as sr


@dataclass
class EndpointFault:
    delay_s: float = 0.0
    reply_delay_s: float = 0.0
    disconnected: bool = False
    corrupt_next: bool = False
    timeout_next: bool = False


@dataclass
class FaultProxy:
    target_host: str
    target_port: int
    host: str = "127.0.0.1"
    port: int = 0
    fault: EndpointFault = field(default_factory=EndpointFault)
    events: list = field(default_factory=list)

    def __post_init__(self):
        self._server = None
        self._tasks: set[asyncio.Task] = set()
        self._writers: set[asyncio.StreamWriter] = set()
        self.frames_forwarded = 0
        self.stats = {"request_frames": 0, "request_bytes": 0, "reply_frames": 0, "reply_bytes": 0}

    async def start(self) -> int:
        self._server = await asyncio.start_server(self._serve, self.host, self.port)
        self.port = self._server.sockets[0].getsockname()[1]
        return self.port

    def _event(self, kind: str, **kw) -> None:
        self.events.append({"type": kind, "at": time.time(), **kw})

    def disconnect(self) -> None:
        """Drop every open connection and refuse new ones until ``reconnect``."""
        self.fault.disconnected = True
        self._event("emulated_disconnection")
        for w in list(self._writers):
            w.close()

    def reconnect(self) -> None:
        self.fault.disconnected = False

    @staticmethod
    async def _read_raw(reader: asyncio.StreamReader) -> tuple[sr.FrameHeader, bytes]:
        head = await reader.readexactly(sr.HEADER_SIZE)
        h = sr.decode_header(head)
        body = await reader.readexactly(h.body_length)
        return h, head + body

    async def _serve(self, cr: asyncio.StreamReader, cw: asyncio.StreamWriter) -> None:
        if self.fault.disconnected:
            self._event("emulated_disconnection", refused=True)
            cw.close()
            return
        try:
            ur, uw = await asyncio.open_connection(self.target_host, self.target_port)
        except OSError:
            cw.close()
            return
        self._writers.update((cw, uw))
        up = asyncio.ensure_future(self._pump_requests(cr, uw))
        down = asyncio.ensure_future(self._pump_replies(ur, cw))
        self._tasks.update((up, down))
        try:
            await asyncio.wait({up, down}, return_when=asyncio.FIRST_COMPLETED)
        finally:
            for t in (up, down):
                t.cancel()
            for w in (cw, uw):
                w.close()
                self._writers.discard(w)
            self._tasks.difference_update((up, down))

    async def _pump_requests(self, cr, uw) -> None:
        try:
            while True:
                h, frame = await self._read_raw(cr)
                if self.fault.disconnected:
                    return
                if self.fault.timeout_next:
                    self.fault.timeout_next = False
                    self._event("emulated_timeout", operation=h.operation.name)
                    continue  # swallowed: the caller never gets a reply
                if self.fault.delay_s:
                    self._event("emulated_wan_delay", delay_s=self.fault.delay_s,
                                operation=h.operation.name)
                    await asyncio.sleep(self.fault.delay_s)
                uw.write(frame)
                await uw.drain()
                self.frames_forwarded += 1
                self.stats["request_frames"] += 1
                self.stats["request_bytes"] += h.body_length
        except (asyncio.IncompleteReadError, ConnectionError, OSError, sr.FrameError):
            return

    async def _pump_replies(self, ur, cw) -> None:
        try:
            while True:
                h, frame = await self._read_raw(ur)
                if self.fault.disconnected:
                    return
                if self.fault.corrupt_next and h.body_length > 0:
                    self.fault.corrupt_next = False
                    b = bytearray(frame)
                    b[-1] ^= 0x01  # last byte of the payload (or of the metadata)
                    frame = bytes(b)
                    self._event("emulated_corrupt_frame", operation=h.operation.name)
                if self.fault.reply_delay_s:
                    await asyncio.sleep(self.fault.reply_delay_s)
                cw.write(frame)
                await cw.drain()
                self.stats["reply_frames"] += 1
                self.stats["reply_bytes"] += h.body_length
        except (asyncio.IncompleteReadError, ConnectionError, OSError, sr.FrameError):
            return

    async def close(self) -> None:
        if self._server is not None:
            self._server.close()
            await self._server.wait_closed()
        for w in list(self._writers):
            w.close()
        for t in list(self._tasks):
            t.cancel()
