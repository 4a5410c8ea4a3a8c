"""Rank liveness over the rendezvous TCP store.

Every rank runs a daemon thread that writes ``hb/<rank>`` = wall time every
``interval`` seconds. ``stale_ranks()`` (any rank, usually rank 0 before each
step) lists ranks whose heartbeat is older than ``timeout`` or missing after
the grace period, and ``check()`` raises ``RankFailure`` for them, so the
scheduler fails in-flight requests on the host instead of entering a
collective that would wait for a dead peer. Device-side waits in the fused
kernels are bounded separately (they record an error code and return).
"""

from __future__ import annotations

import threading
import time


class RankFailure(RuntimeError):
    def __init__(self, ranks):
        super().__init__(f"ranks not responding: {sorted(ranks)}")
        self.ranks = sorted(ranks)


class Heartbeat:
    def __init__(self, store, rank: int, world: int, interval: float = 0.5, timeout: float = 5.0,
                 prefix: str = "hb"):
        self.store, self.rank, self.world = store, rank, world
        self.interval, self.timeout, self.prefix = interval, timeout, prefix
        self._stop = threading.Event()
        self._t = None
        self.started = time.time()

    def _key(self, r):
        return f"{self.prefix}/{r}"

    def beat(self):
        self.store.set(self._key(self.rank), repr(time.time()))

    def _run(self):
        while not self._stop.is_set():
            try:
                self.beat()
            except Exception:  # store gone: the rendezvous owner died; nothing else to do
                return
            self._stop.wait(self.interval)

    def start(self):
        if self._t is None:
            self.beat()
            self._t = threading.Thread(target=self._run, name=f"heartbeat-{self.rank}", daemon=True)
            self._t.start()
        return self

    def stop(self):
        self._stop.set()
        if self._t is not None:
            self._t.join(timeout=5)
            self._t = None

    def last_seen(self, r):
        try:
            if not self.store.check([self._key(r)]):
                return None
            return float(self.store.get(self._key(r)).decode())
        except Exception:
            return None

    def stale_ranks(self, now: float = None) -> list:
        now = now or time.time()
        bad = []
        for r in range(self.world):
            if r == self.rank:
                continue
            t = self.last_seen(r)
            if t is None:
                if now - self.started > self.timeout:
                    bad.append(r)
            elif now - t > self.timeout:
                bad.append(r)
        return bad

    def check(self):
        bad = self.stale_ranks()
        if bad:
            raise RankFailure(bad)
