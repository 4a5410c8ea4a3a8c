"""Error classification, retry and OOM recovery (reference: core/resilience.py:19-202)."""

from __future__ import annotations

import functools
import gc
import logging
import time

_log = logging.getLogger(__name__)

_TRANSIENT_PATTERNS = [
    "connection reset", "connection refused", "timed out", "timeout", "temporarily unavailable",
    "broken pipe", "cuda error: an illegal memory access",  # never retried: see is_recoverable
    "resource temporarily", "503", "502", "429",
]


def is_oom(exc) -> bool:
    msg = str(exc).lower()
    return "out of memory" in msg or type(exc).__name__ in ("OutOfMemoryError",)


def is_recoverable(exc) -> bool:
    """Transient errors worth a retry. A CUDA fault is never recoverable."""
    msg = str(exc).lower()
    if "illegal memory access" in msg or "device-side assert" in msg:
        return False
    if is_oom(exc):
        return True
    return any(p in msg for p in _TRANSIENT_PATTERNS)


def retry_with_backoff(max_retries=3, initial_delay=1.0, backoff_factor=2.0, exceptions=(Exception,)):
    def deco(fn):
        @functools.wraps(fn)
        def wrapper(*a, **kw):
            delay = initial_delay
            for attempt in range(max_retries + 1):
                try:
                    return fn(*a, **kw)
                except exceptions as e:  # noqa: PERF203
                    if attempt == max_retries or not is_recoverable(e):
                        raise
                    _log.warning("retry %d/%d after %s", attempt + 1, max_retries, e)
                    time.sleep(delay)
                    delay *= backoff_factor
        return wrapper
    return deco


class engine_recovery:
    """Context manager: on an OOM inside the block, free cached device memory
    and swallow nothing (the caller decides whether to retry)."""

    def __init__(self, engine):
        self.engine = engine
        self.oom = False

    def __enter__(self):
        return self

    def __exit__(self, exc_type, exc, tb):
        if exc is not None and is_oom(exc):
            self.oom = True
            self._free_vram()
        return False

    def _free_vram(self):
        gc.collect()
        try:
            import torch
            if torch.cuda.is_available():
                torch.cuda.empty_cache()
        except Exception:
            pass
        cleanup = getattr(self.engine, "periodic_cleanup", None)
        if cleanup:
            cleanup()


def generate_with_recovery(engine, messages, max_tokens, temperature, max_attempts=3, **kwargs):
    """generate_streaming with OOM recovery: each retry halves max_tokens and
    compresses the history (reference :149-202)."""
    from b200serve.core.inference import compress_history
    msgs, mt = list(messages), max_tokens
    for attempt in range(max_attempts):
        rec = engine_recovery(engine)
        try:
            with rec:
                return engine.generate_streaming(msgs, mt, temperature, **kwargs)
        except Exception as e:
            if not rec.oom or attempt == max_attempts - 1:
                raise
            mt = max(64, mt // 2)
            msgs = compress_history(msgs, max(2, (len(msgs) - 1) // 2))
            _log.warning("OOM: retry with max_tokens=%d, %d messages", mt, len(msgs))
    return ""
