"""Coordinator runtime: idempotent lifecycle owner of the coordinator's services.

Components (durable state, worker registry, deployment manager, control server,
background sweeps) are started in order; if one fails, the ones already started are
stopped in reverse and the error is re-raised (partial-start rollback).  ``start``
and ``stop`` are idempotent; ``stop`` never raises for a component that failed to
stop, it records the error.

Reference: si/coordinator/runtime.py:66.
"""
from __future__ import annotations

import asyncio
import inspect
from dataclasses import dataclass, field


@dataclass
class Component:
    name: str
    start: object                 # callable (sync or async)
    stop: object | None = None
    started: bool = False


@dataclass
class CoordinatorRuntime:
    components: list[Component] = field(default_factory=list)
    running: bool = False
    errors: list[tuple[str, str]] = field(default_factory=list)

    def add(self, name: str, start, stop=None) -> None:
        self.components.append(Component(name, start, stop))

    @staticmethod
    async def _call(fn):
        r = fn()
        if inspect.isawaitable(r):
            await r

    async def start(self) -> None:
        if self.running:
            return
        for c in self.components:
            try:
                await self._call(c.start)
                c.started = True
            except Exception:
                await self._stop_started()
                raise
        self.running = True

    async def _stop_started(self) -> None:
        for c in reversed(self.components):
            if not c.started:
                continue
            try:
                if c.stop is not None:
                    await self._call(c.stop)
            except Exception as exc:  # noqa: BLE001 - keep stopping the rest
                self.errors.append((c.name, f"{type(exc).__name__}: {exc}"))
            c.started = False

    async def stop(self) -> None:
        await self._stop_started()
        self.running = False

    def run(self, main) -> None:
        """Start, run ``main()`` (coroutine function), always stop."""
        async def body():
            await self.start()
            try:
                await main()
            finally:
                await self.stop()
        asyncio.run(body())
