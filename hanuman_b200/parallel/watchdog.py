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
                    try:
                        v = self.store.get(self._key(r)).decode()
                        ts = float(v.split(":")[1])
                    except Exception:
                        ts = 0.0
                    if now - ts > self.timeout_s:
                        dead.append(r)
                self.dead = dead
            except Exception:
                pass

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
