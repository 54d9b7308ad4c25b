"""Memory pressure levels and actions (reference ``src/strix/vram_pressure.rs``:
Green < 60 % <= Yellow < 75 % <= Orange < 85 % <= Red < 95 % <= Critical of the budget
(total minus a safety margin), with recommended actions per level).

On a B200 the weights and the KV pool are allocated once, so the memory that moves is the
KV pool's block usage. ``KvPressureController`` evaluates that every scheduler step and acts
on the engine: from Orange on it returns prefix-cache blocks to the pool, from Red on it
stops admitting new requests for the step, and at Critical it empties the prefix cache and
preempts (swaps out) the most recently admitted running request.
"""
from __future__ import annotations

import enum
from dataclasses import dataclass


class PressureLevel(enum.IntEnum):
    GREEN = 0
    YELLOW = 1
    ORANGE = 2
    RED = 3
    CRITICAL = 4

    def __str__(self) -> str:
        return {0: "Green (<60%)", 1: "Yellow (60-75%)", 2: "Orange (75-85%)", 3: "Red (85-95%)",
                4: "Critical (>=95%)"}[int(self)]


@dataclass(frozen=True)
class PressureAction:
    kind: str                       # continue / reduce_prefetch / evict_class / suspend_prefetch /
    value: int = 0                  # compress_kv / emergency_evict / set_flight_slot


class VramPressureManager:
    def __init__(self, total_bytes: int, safety_margin: int = 0, default_prefetch_window: int = 2):
        self.total = int(total_bytes)
        self.safety_margin = int(safety_margin)
        self.default_prefetch_window = default_prefetch_window
        self.budget = max(0, self.total - self.safety_margin)

    def utilisation(self, used: int) -> float:
        return 1.0 if self.budget == 0 else used / self.budget

    def evaluate(self, used: int) -> PressureLevel:
        if self.budget == 0:
            return PressureLevel.CRITICAL
        r = used / self.budget
        if r >= 0.95:
            return PressureLevel.CRITICAL
        if r >= 0.85:
            return PressureLevel.RED
        if r >= 0.75:
            return PressureLevel.ORANGE
        if r >= 0.60:
            return PressureLevel.YELLOW
        return PressureLevel.GREEN

    def recommended_actions(self, level: PressureLevel) -> list[PressureAction]:
        if level == PressureLevel.GREEN:
            return [PressureAction("continue")]
        if level == PressureLevel.YELLOW:
            return [PressureAction("reduce_prefetch", max(1, self.default_prefetch_window // 2))]
        if level == PressureLevel.ORANGE:
            return [PressureAction("evict_class", 2), PressureAction("compress_kv")]
        if level == PressureLevel.RED:
            return [PressureAction("evict_class", 1), PressureAction("suspend_prefetch"), PressureAction("compress_kv")]
        return [PressureAction("emergency_evict")]

    @staticmethod
    def recommended_flight_slot_size(level: PressureLevel) -> int:
        return {PressureLevel.GREEN: 512 << 20, PressureLevel.YELLOW: 256 << 20,
                PressureLevel.ORANGE: 128 << 20}.get(level, 64 << 20)


def kv_cache_budget(context_len: int, n_kv_heads: int, head_dim: int, n_layers: int, dtype_bytes: int = 2) -> int:
    return 2 * context_len * n_kv_heads * head_dim * n_layers * dtype_bytes


class KvPressureController:
    """Applies pressure actions to an ``Engine`` from its KV pool usage."""

    def __init__(self, engine, safety_blocks: int = 0):
        self.eng = engine
        alloc = engine.seqs.allocator
        self.mgr = VramPressureManager(alloc.total_blocks, safety_blocks)
        self.level = PressureLevel.GREEN
        self.history: list[PressureLevel] = []
        self.evicted_blocks = 0
        self.preempted = 0

    def used(self) -> int:
        return self.eng.seqs.allocator.num_used_blocks()

    def tick(self) -> PressureLevel:
        """Evaluate and act; returns the level before acting. Sets ``admit_paused`` on the
        engine while the pool is at Red or above."""
        eng = self.eng
        lvl = self.mgr.evaluate(self.used())
        self.level = lvl
        self.history.append(lvl)
        pc = eng.prefix_cache
        if lvl >= PressureLevel.ORANGE and pc is not None:
            target = self.used() - int(0.70 * self.mgr.budget)
            if lvl == PressureLevel.CRITICAL:
                target = pc.size()
            if target > 0:
                self.evicted_blocks += pc.evict_until(target)
        eng.admit_paused = lvl >= PressureLevel.RED
        if lvl == PressureLevel.CRITICAL and eng.swap is not None and len(eng.running) > 1:
            if eng.preempt_latest():
                self.preempted += 1
        return lvl
