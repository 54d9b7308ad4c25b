"""Multi-rank serving: one HTTP front end, every tensor-parallel rank stepping in lockstep
(reference ``DistributedDispatcher`` / ``serve_follower``, ``src/dispatcher.rs:130-200``).

Rank 0 owns HTTP and the scheduler input: new requests (and embedding calls) arrive on its
dispatcher queue. Every scheduler tick it broadcasts, on a CPU (gloo) control group, the
list of items admitted this tick plus a digest of its engine state (step count, running /
waiting counts); every rank then admits the same items in the same order and, when its
engine has unfinished work, runs one ``Engine.step``. Engines are built identically and
scheduling is deterministic, so all ranks hold the same batch, block tables and positions,
and the step's NCCL / peer-memory collectives line up. Tokens are sampled on every rank
from the same all-gathered logits with the same Philox seed, so they agree without another
message; only rank 0 streams them to clients.

The reference forwards each request's config to the followers, which run the request
to completion one at a time; here followers mirror a continuous batch. Idle ticks (nothing
admitted, nothing running) are sent at most every ``idle_tick_s`` so followers never sit
in one broadcast long enough for the process-group timeout to end them. A follower that
sees a different state digest than rank 0 raises: a diverged rank must not join the next
collective with other inputs.
"""
from __future__ import annotations

import queue
import time

import torch.distributed as dist

from .dispatcher import EngineDispatcher, FinishReason


class StateDivergence(RuntimeError):
    pass


def _digest(eng) -> tuple:
    return (eng.step_count, len(eng.running), len(eng.waiting), len(getattr(eng, "swapped", [])))


class DistributedDispatcher(EngineDispatcher):
    """``EngineDispatcher`` whose engine loop is mirrored on every rank of ``group``.

    Rank 0: construct it and serve HTTP with it (its ``generate`` / ``embed`` as usual).
    Other ranks: construct it and call ``serve_follower()``, which returns on shutdown."""

    STOP = "__stop__"

    def __init__(self, engine, model_name: str = "air-rs", group=None, health=None,
                 idle_tick_s: float = 1.0):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.idle_tick_s = idle_tick_s
        self.ticks = 0
        self.history: dict[int, list[int]] = {}     # rid -> output ids of finished requests
        if self.rank == 0:
            super().__init__(engine, model_name, health)
        else:
            # followers run the loop on the caller's thread (serve_follower), no queue
            self.engine, self.model_name, self.health = engine, model_name, health
            self.errors = 0
            self.requests_served = 0
            self._texts = None
            self._thread = None

    # -- control channel ------------------------------------------------------------------
    def _bcast(self, msg):
        box = [msg]
        dist.broadcast_object_list(box, src=0, group=self.group)
        self.ticks += 1
        return box[0]

    @staticmethod
    def _wire(item):
        """What followers need of a queued item (callbacks stay on rank 0)."""
        if item[0] == "embed":
            return ("embed", item[1])
        return ("gen", item[1])

    def _apply(self, wire_items):
        """Follower side of _admit: same admission, no client callbacks."""
        noop = lambda *a, **k: None
        for it in wire_items:
            if it[0] == "embed":
                try:
                    self.engine.embed(it[1])
                except Exception:
                    pass
            else:
                self._admit(("gen", it[1], noop, noop))

    def _step_once(self):
        eng = self.engine
        if not eng.has_unfinished():
            return
        try:
            if self.health is not None:
                self.health.check()
            eng.step()
        except Exception as e:
            self.errors += 1
            for r in list(eng.running) + list(eng.waiting) + list(getattr(eng, "swapped", [])):
                cb = getattr(r, "_on_done", None)
                r._on_done = None
                eng.abort(r.rid)
                if cb:
                    cb(FinishReason.ERROR, str(e))

    # -- rank 0 -----------------------------------------------------------------------------
    def _loop(self):
        eng = self.engine
        last = time.monotonic()
        while True:
            stop = self._stop.is_set()
            items = []
            if not stop:
                try:
                    wait = 0.0 if eng.has_unfinished() else min(0.05, self.idle_tick_s)
                    item = self._submit.get(timeout=wait) if wait > 0 else self._submit.get_nowait()
                    while item is not None:
                        items.append(item)
                        item = self._submit.get_nowait()
                except queue.Empty:
                    pass
                stop = self._stop.is_set()
            items = [it for it in items if it is not None]
            now = time.monotonic()
            if not stop and not items and not eng.has_unfinished() and now - last < self.idle_tick_s:
                continue
            last = now
            self._bcast((_digest(eng), [self._wire(it) for it in items], stop))
            if stop:
                return
            for it in items:
                self._admit(it)
            self._step_once()
            for rid, r in eng.finished.items():
                self.history[rid] = list(r.output_ids)
            self._reap()

    # -- followers --------------------------------------------------------------------------
    def serve_follower(self):
        """Mirror rank 0's engine loop until it shuts down."""
        if self.rank == 0:
            raise RuntimeError("serve_follower() runs on ranks other than 0")
        eng = self.engine
        while True:
            digest, items, stop = self._bcast(None)
            if stop:
                return
            if digest != _digest(eng):
                raise StateDivergence(f"rank {self.rank}: engine state {_digest(eng)} != rank 0's {digest}")
            self._apply(items)
            self._step_once()
            for rid, r in eng.finished.items():
                self.history[rid] = list(r.output_ids)
            eng.finished.clear()

    def shutdown(self):
        if self.rank == 0:
            super().shutdown()
