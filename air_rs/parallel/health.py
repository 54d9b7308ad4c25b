"""Rank failure detection (reference: only transfer deadlines, ``src/pd_disagg.rs:290-312``;
no heartbeats there). Each rank runs a heartbeat thread that bumps a counter in a shared
``torch.distributed`` store; a monitor reports ranks whose counter stopped moving for longer
than ``timeout``, or that announced an orderly exit. The engine checks ``dead_ranks()``
between steps and fails pending work with ``CommTimeout`` instead of entering a collective
that would wait for a dead peer. No GPU is involved: failures are injected on the host
(an exception, an early exit, a stalled heartbeat).
"""
from __future__ import annotations

import threading
import time


class CommTimeout(RuntimeError):
    pass


class Heartbeat:
    def __init__(self, store, rank: int, world: int, interval: float = 0.1, timeout: float = 1.0,
                 prefix: str = "air_hb"):
        self.store, self.rank, self.world = store, rank, world
        self.interval, self.timeout, self.prefix = interval, timeout, prefix
        self._stop = threading.Event()
        self._paused = threading.Event()
        self._thread = threading.Thread(target=self._beat, daemon=True)
        self._seen: dict[int, tuple[int, float]] = {}

    def _key(self, r, kind="beat"):
        return f"{self.prefix}/{kind}/{r}"

    def start(self) -> "Heartbeat":
        self.store.set(self._key(self.rank, "exit"), "0")
        self._thread.start()
        return self

    def _beat(self):
        while not self._stop.is_set():
            if not self._paused.is_set():
                self.store.add(self._key(self.rank), 1)
            self._stop.wait(self.interval)

    def pause(self):
        """Fault injection: stop beating while the process stays alive (a hung rank)."""
        self._paused.set()

    def stop(self, orderly: bool = True):
        self._stop.set()
        if orderly:
            self.store.set(self._key(self.rank, "exit"), "1")

    def dead_ranks(self) -> list[int]:
        now = time.monotonic()
        dead = []
        for r in range(self.world):
            if r == self.rank:
                continue
            try:
                exited = self.store.get(self._key(r, "exit")) == b"1"
            except Exception:
                exited = False
            n = self.store.add(self._key(r), 0)
            last = self._seen.get(r)
            if last is None or last[0] != n:
                self._seen[r] = (n, now)
            elif now - last[1] > self.timeout:
                dead.append(r)
                continue
            if exited:
                dead.append(r)
        return dead

    def check(self):
        d = self.dead_ranks()
        if d:
            raise CommTimeout(f"ranks {d} stopped responding")
