"""ModelMux (reference ``src/model_mux.rs``): several engines behind one loop, stepped in an
interleaved tick so each model's continuous batch advances fairly, with per-model prefix
caches (``Engine(prefix_cache=True)``) and events for submit / token / finish.
"""
from __future__ import annotations

import enum
from dataclasses import dataclass


class MuxEventKind(str, enum.Enum):
    SUBMITTED = "submitted"
    TOKEN = "token"
    FINISHED = "finished"


@dataclass
class MuxEvent:
    kind: MuxEventKind
    model: str
    rid: int
    token: int | None = None


class ModelMux:
    def __init__(self):
        self.engines: dict[str, object] = {}
        self.events: list[MuxEvent] = []
        self._order: list[str] = []
        self._next = 0

    def add_model(self, name: str, engine):
        self.engines[name] = engine
        self._order.append(name)

    def submit(self, model: str, prompt_ids: list[int], params=None) -> int:
        eng = self.engines[model]
        rid = eng.add_request(prompt_ids, params)
        self.events.append(MuxEvent(MuxEventKind.SUBMITTED, model, rid))
        return rid

    def tick(self) -> int:
        """One step of the next model that has work (round robin); returns tokens produced."""
        for _ in range(len(self._order)):
            name = self._order[self._next % len(self._order)]
            self._next += 1
            eng = self.engines[name]
            if not eng.has_unfinished():
                continue
            before = set(eng.finished)
            produced = eng.step()
            for rid, tok in produced:
                self.events.append(MuxEvent(MuxEventKind.TOKEN, name, rid, tok))
            for rid in set(eng.finished) - before:
                self.events.append(MuxEvent(MuxEventKind.FINISHED, name, rid))
            return len(produced)
        return 0

    def run_until_idle(self, max_ticks: int = 1 << 20):
        for _ in range(max_ticks):
            if not any(e.has_unfinished() for e in self.engines.values()):
                return
            self.tick()
