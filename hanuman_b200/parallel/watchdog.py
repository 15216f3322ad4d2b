"""Host-side failure detection for data-parallel training.

Every rank publishes a heartbeat (step counter + wall time) in the
process-group store from a daemon thread; the same thread reads the peers'
heartbeats and flags a peer whose heartbeat is older than ``timeout_s``.  The
training loop calls :meth:`Watchdog.check` between steps (never while its own
kernels or collectives are in flight) and gets a :class:`PeerFailure` naming
the silent ranks, instead of blocking in the next collective.  Device-side
waits are bounded independently (the status word of the native kernels).
"""
from __future__ import annotations

import threading
import time


class PeerFailure(RuntimeError):
    pass


class Watchdog:
    def __init__(self, store, rank: int, world: int, timeout_s: float = 30.0,
                 interval_s: float = 1.0, prefix: str = "hb_heartbeat"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.interval_s, self.prefix = timeout_s, interval_s, prefix
        self.step = 0
        self.dead: list[int] = []
        self._t0 = time.time()   # a peer with no heartbeat yet counts from here
        self._stop = threading.Event()
        self._t = threading.Thread(target=self._loop, daemon=True)
        self._beat()
        self._t.start()

    def _key(self, r):
        return f"{self.prefix}/{r}"

    def _beat(self):
        self.store.set(self._key(self.rank), f"{self.step}:{time.time():.3f}")

    def _loop(self):
        while not self._stop.wait(self.interval_s):
            try:
                self._beat()
                now = time.time()
                dead = []
                for r in range(self.world):
                    if r == self.rank:
                        continue
                    ts = self._peer_time(r)
                    if now - ts > self.timeout_s:
                        dead.append(r)
                self.dead = dead
            except Exception:
                pass

    def _peer_time(self, r) -> float:
        """Wall time of peer r's last heartbeat.  ``store.check`` does not
        block, so a peer that never wrote one (it died before its first beat)
        costs no store timeout: it counts from this watchdog's start and is
        reported once ``timeout_s`` has passed."""
        key = self._key(r)
        try:
            if not self.store.check([key]):
                return self._t0
            return float(self.store.get(key).decode().split(":")[1])
        except Exception:
            return self._t0

    def tick(self, step: int):
        self.step = step

    def check(self):
        """Raise PeerFailure when any peer has stopped beating."""
        if self.dead:
            raise PeerFailure(f"rank {self.rank}: no heartbeat from ranks {self.dead} "
                              f"for more than {self.timeout_s:.0f} s")

    def close(self):
        self._stop.set()
        self._t.join(timeout=5)
