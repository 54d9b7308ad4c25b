"""Tensor residency scoring, a priority I/O engine and a residency scheduler (reference
``src/strix/score.rs``: R(t, tau) = w_u U + w_p P + w_s S + w_c C with a sigmoid urgency of
the distance to next use, exponential recency, log-scaled eviction stickiness and size cost;
``src/strix/io_engine.rs``: priority queue of file reads by tensor class with a bounded number
in flight; ``src/strix/scheduler.rs``: keep the highest-scoring tensors within the budget).

``IoEngine`` does the reads: a pool of threads issues ``os.pread`` of (offset, size) ranges
of a checkpoint into pinned host buffers, highest priority first, so a cold start or a
streamed model pulls the tensors it needs next before the ones it needs later.
"""
from __future__ import annotations

import enum
import heapq
import itertools
import math
import os
import threading
import time
from dataclasses import dataclass, field

import torch


@dataclass
class ScoreWeights:
    urgency: float = 0.45
    predictive: float = 0.30
    sticky: float = 0.15
    cost: float = 0.10

    def sum(self) -> float:
        return self.urgency + self.predictive + self.sticky + self.cost


def urgency(distance_layers: int, prefetch_window: int) -> float:
    """1 / (1 + exp(0.8 (d - W))): ~1 inside the prefetch window, 0.5 at its edge."""
    if prefetch_window == 0:
        return 1.0 if distance_layers == 0 else 0.0
    return 1.0 / (1.0 + math.exp(0.8 * (distance_layers - prefetch_window)))


def predictive(last_access_step: int, current_step: int, decay: float = 0.1) -> float:
    if current_step <= last_access_step:
        return 1.0
    return math.exp(-decay * (current_step - last_access_step))


def sticky(eviction_count: int) -> float:
    """ln(1 + e) / ln(21), capped at 1: tensors evicted often get a bonus to stay."""
    if eviction_count <= 0:
        return 0.0
    return min(1.0, math.log1p(eviction_count) / math.log(21.0))


def cost(size_bytes: int, max_tensor_bytes: int) -> float:
    return 0.0 if max_tensor_bytes <= 0 else min(1.0, size_bytes / max_tensor_bytes)


def residency_score(w: ScoreWeights, u: float, p: float, s: float, c: float) -> float:
    return min(1.0, max(0.0, w.urgency * u + w.predictive * p + w.sticky * s + w.cost * c))


class TensorClass(str, enum.Enum):
    A = "A"     # always resident (embeddings, norms, LM head)
    B = "B"     # layer weights
    C = "C"     # drafter / auxiliary
    D = "D"     # cold (rarely used experts)


class IoPriority(enum.IntEnum):
    CRITICAL = 0
    HIGH = 1
    NORMAL = 2
    LOW = 3

    @classmethod
    def from_class(cls, tc: TensorClass, within_window: bool) -> "IoPriority":
        if tc == TensorClass.A:
            return cls.CRITICAL
        if tc in (TensorClass.B, TensorClass.C) and within_window:
            return cls.HIGH
        if tc == TensorClass.B:
            return cls.NORMAL
        return cls.LOW


@dataclass
class IoRequest:
    tensor_id: str
    file_offset: int
    size: int
    priority: IoPriority = IoPriority.NORMAL


@dataclass
class IoCompletion:
    ticket: int
    tensor_id: str
    data: torch.Tensor          # uint8 [size], pinned when CUDA is available
    elapsed_s: float
    error: str | None = None


class IoEngine:
    """Prioritised reads of byte ranges of one file by ``workers`` threads, at most
    ``capacity`` in flight."""

    def __init__(self, path: str, capacity: int = 8, workers: int = 4, pin: bool | None = None,
                 start_paused: bool = False):
        self.path = path
        self.fd = os.open(path, os.O_RDONLY)
        self.capacity = capacity
        self.pin = torch.cuda.is_available() if pin is None else pin
        self._q: list = []
        self._tickets = itertools.count(1)
        self._seq = itertools.count()
        self._cv = threading.Condition()
        self._inflight = 0
        self._done: list[IoCompletion] = []
        self._closed = False
        self._paused = start_paused
        self._threads = [threading.Thread(target=self._work, daemon=True) for _ in range(max(1, workers))]
        for t in self._threads:
            t.start()

    def submit(self, req: IoRequest) -> int:
        t = next(self._tickets)
        with self._cv:
            heapq.heappush(self._q, (int(req.priority), next(self._seq), t, req))
            self._cv.notify()
        return t

    def _work(self):
        while True:
            with self._cv:
                while not self._closed and (self._paused or not self._q or self._inflight >= self.capacity):
                    self._cv.wait()
                if self._closed:
                    return
                _, _, ticket, req = heapq.heappop(self._q)
                self._inflight += 1
            t0 = time.perf_counter()
            err = None
            buf = torch.empty(req.size, dtype=torch.uint8, pin_memory=self.pin)
            try:
                mv = memoryview(buf.numpy())
                got = 0
                while got < req.size:
                    n = os.preadv(self.fd, [mv[got:]], req.file_offset + got)
                    if n <= 0:
                        raise EOFError(f"short read at {req.file_offset + got}")
                    got += n
            except Exception as e:
                err = f"{type(e).__name__}: {e}"
            with self._cv:
                self._inflight -= 1
                self._done.append(IoCompletion(ticket, req.tensor_id, buf, time.perf_counter() - t0, err))
                self._cv.notify_all()

    def resume(self):
        with self._cv:
            self._paused = False
            self._cv.notify_all()

    def poll(self) -> list[IoCompletion]:
        with self._cv:
            out, self._done = self._done, []
        return out

    def wait_all(self, timeout: float = 60.0) -> list[IoCompletion]:
        end = time.monotonic() + timeout
        with self._cv:
            while (self._q or self._inflight) and time.monotonic() < end:
                self._cv.wait(timeout=0.05)
        return self.poll()

    def queued_count(self) -> int:
        with self._cv:
            return len(self._q)

    def in_flight_count(self) -> int:
        with self._cv:
            return self._inflight

    def close(self):
        with self._cv:
            self._closed = True
            self._cv.notify_all()
        for t in self._threads:
            t.join(timeout=5)
        os.close(self.fd)


@dataclass
class TrackedTensor:
    tensor_id: str
    size: int
    cls: TensorClass = TensorClass.B
    layer: int = 0
    last_access: int = 0
    evictions: int = 0
    resident: bool = False


@dataclass
class ResidencyScheduler:
    """Keeps the highest-scoring tensors resident within ``budget_bytes`` (class A always)."""
    budget_bytes: int
    prefetch_window: int = 2
    weights: ScoreWeights = field(default_factory=ScoreWeights)
    tensors: dict = field(default_factory=dict)
    step: int = 0

    def register(self, t: TrackedTensor):
        self.tensors[t.tensor_id] = t

    def score(self, t: TrackedTensor, current_layer: int, n_layers: int) -> float:
        if t.cls == TensorClass.A:
            return 1.0
        dist = (t.layer - current_layer) % max(1, n_layers)
        mx = max(x.size for x in self.tensors.values())
        return residency_score(self.weights, urgency(dist, self.prefetch_window),
                               predictive(t.last_access, self.step), sticky(t.evictions), cost(t.size, mx))

    def tick(self, current_layer: int, n_layers: int) -> tuple[list[str], list[str]]:
        """(to load, to evict) for the new resident set at ``current_layer``."""
        self.step += 1
        ranked = sorted(self.tensors.values(), key=lambda t: -self.score(t, current_layer, n_layers))
        keep, used = set(), 0
        for t in ranked:
            if t.cls == TensorClass.A or used + t.size <= self.budget_bytes:
                keep.add(t.tensor_id)
                used += t.size
        load, evict = [], []
        for t in self.tensors.values():
            if t.tensor_id in keep and not t.resident:
                load.append(t.tensor_id)
                t.resident = True
            elif t.tensor_id not in keep and t.resident:
                evict.append(t.tensor_id)
                t.resident = False
                t.evictions += 1
            if t.layer == current_layer:
                t.last_access = self.step
        return load, evict


# ---------------------------------------------------------------------------------------
# Memory budget (native) and cold boot (reference src/strix/arena.rs, src/strix/ram_pool.rs,
# src/strix/cold_boot.rs)
# ---------------------------------------------------------------------------------------

def vram_arena(total_bytes: int, safety_margin: int = 0):
    """The native first-fit VRAM budget arena (``air_rs._host.VramArena``): offsets within a
    budget, alignment, coalescing on free, and a round-robin ring of prefetch flight slots."""
    from .. import _host
    return _host.VramArena(total_bytes, safety_margin)


def ram_pool(max_bytes: int):
    """The native host staging-buffer pool (``air_rs._host.RamPool``), power-of-two classes."""
    from .. import _host
    return _host.RamPool(max_bytes)


@dataclass
class ColdBootStep:
    name: str
    target: str          # "pinned" | "hot" | "warm" | "cold"
    phase: int
    size_bytes: int


@dataclass
class ColdBootPlan:
    steps: list
    phase_bytes: dict    # phase -> bytes
    skipped: int

    @property
    def total_transfer_bytes(self) -> int:
        """Bytes moved at boot: phases 1-3 (pin, first layers hot, the rest staged in RAM)."""
        return sum(self.phase_bytes.get(p, 0) for p in (1, 2, 3))

    @property
    def critical_path_bytes(self) -> int:
        """Bytes that must land before the first token: phases 1 and 2."""
        return sum(self.phase_bytes.get(p, 0) for p in (1, 2))

    def estimate_seconds(self, mb_per_s: float) -> float:
        return float("inf") if mb_per_s <= 0 else self.total_transfer_bytes / 2**20 / mb_per_s

    def estimate_ttft_seconds(self, mb_per_s: float) -> float:
        return float("inf") if mb_per_s <= 0 else self.critical_path_bytes / 2**20 / mb_per_s


def plan_cold_boot(tensors, prefetch_window: int) -> ColdBootPlan:
    """Order a model's first load by tensor class (reference ``src/strix/cold_boot.rs:76-170``).

    ``tensors``: iterable of (name, TensorClass, layer or None, size_bytes). Phase 1 pins
    class A (embeddings, norms, LM head); phase 2 makes class-B layers below
    ``prefetch_window`` hot in HBM, in layer order; phase 3 stages the other class-B layers
    in host RAM (warm); phase 4 leaves class C on disk (cold); class D is skipped."""
    steps, pb, skipped = [], {}, 0
    items = list(tensors)

    def add(name, target, phase, size):
        steps.append(ColdBootStep(name, target, phase, size))
        pb[phase] = pb.get(phase, 0) + size

    for name, tc, layer, size in items:
        if tc == TensorClass.A:
            add(name, "pinned", 1, size)
    b = sorted((x for x in items if x[1] == TensorClass.B),
               key=lambda x: x[2] if x[2] is not None else 1 << 60)
    for name, tc, layer, size in b:
        if layer is not None and layer < prefetch_window:
            add(name, "hot", 2, size)
        else:
            add(name, "warm", 3, size)
    for name, tc, layer, size in items:
        if tc == TensorClass.C:
            add(name, "cold", 4, size)
        elif tc == TensorClass.D:
            skipped += 1
    return ColdBootPlan(steps, pb, skipped)
