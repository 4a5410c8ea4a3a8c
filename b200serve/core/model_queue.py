"""Model queue (reference: core/model_queue.py:55-462).

The reference serialises every request behind one asyncio lock because its
runtimes serve one request at a time. This engine batches requests
continuously, so the queue only serialises *model switches*: a request for
the loaded model enters the engine's scheduler at once, a request for
another model waits for in-flight requests to drain, then the engine is
swapped. Busy checks (e.g. an agent run holding the engine) and idle-shrink
are kept.
"""

from __future__ import annotations

import asyncio
import logging
import os
import time

_log = logging.getLogger(__name__)

IDLE_SHRINK_SEC = int(os.environ.get("ARTIFEX_IDLE_SHRINK_SEC", "600"))


class ModelBusyError(RuntimeError):
    """Raised when a switch is refused because something holds the engine."""


class ModelQueue:
    def __init__(self):
        self._lock = asyncio.Lock()           # held only while switching
        self._current_model = None
        self._current_backend = None
        self._ctx_tier = None
        self._switch_count = 0
        self._served = 0
        self._in_flight = 0
        self._busy_checks = []
        self._unload_fns = []
        self._last_activity = time.time()
        self._drained = None

    # ----- hooks -----
    def register_transformers_unload(self, fn):
        """Kept name: register a callable that unloads the active engine."""
        self._unload_fns.append(fn)

    register_engine_unload = register_transformers_unload

    def register_busy_check(self, fn):
        self._busy_checks.append(fn)

    def busy_reason(self):
        for fn in self._busy_checks:
            try:
                r = fn()
            except Exception:
                r = None
            if r:
                return r
        return None

    def note_activity(self):
        self._last_activity = time.time()

    @property
    def current_model(self):
        return self._current_model

    @property
    def current_ctx_tier(self):
        return self._ctx_tier

    @property
    def stats(self) -> dict:
        return {"current_model": self._current_model, "current_backend": self._current_backend,
                "in_flight": self._in_flight, "served": self._served,
                "switch_count": self._switch_count, "ctx_tier": self._ctx_tier,
                "idle_s": round(time.time() - self._last_activity, 1)}

    # ----- request accounting -----
    def request_started(self):
        self._in_flight += 1
        self.note_activity()

    def request_finished(self):
        self._in_flight = max(0, self._in_flight - 1)
        self._served += 1
        self.note_activity()
        if self._in_flight == 0 and self._drained is not None:
            self._drained.set()

    async def _wait_drained(self, timeout=600.0):
        if self._in_flight == 0:
            return
        self._drained = asyncio.Event()
        try:
            await asyncio.wait_for(self._drained.wait(), timeout)
        finally:
            self._drained = None

    async def switch_if_needed(self, model, backend=None, ctx_tier=None) -> bool:
        """Make ``model`` the served model. Returns True if a switch happened."""
        if model == self._current_model and backend in (None, self._current_backend) \
                and (ctx_tier is None or self._ctx_tier is None or ctx_tier <= self._ctx_tier):
            return False
        async with self._lock:
            if self._current_model is not None:
                reason = self.busy_reason()
                if reason:
                    raise ModelBusyError(reason)
                await self._wait_drained()
                await self.unload_current()
                self._switch_count += 1
            self._current_model = model
            self._current_backend = backend or self._current_backend
            self._ctx_tier = ctx_tier
            self.note_activity()
            return True

    async def unload_current(self):
        for fn in self._unload_fns:
            try:
                r = fn()
                if asyncio.iscoroutine(r):
                    await r
            except Exception as e:  # an unload failure must not wedge the queue
                _log.warning("unload hook failed: %s", e)

    def idle_for(self) -> float:
        return time.time() - self._last_activity

    async def idle_shrink_once(self):
        """Unload the engine when nothing ran for IDLE_SHRINK_SEC."""
        if self._in_flight == 0 and self._current_model and self.idle_for() > IDLE_SHRINK_SEC:
            async with self._lock:
                await self.unload_current()
                self._current_model = None
                return True
        return False


_queue = None


def get_model_queue() -> ModelQueue:
    global _queue
    if _queue is None:
        _queue = ModelQueue()
    return _queue
