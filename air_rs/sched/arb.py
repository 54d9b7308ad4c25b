"""Adaptive Resonance Batching (reference ``src/batching/arb.rs``) and an Orca/Sarathi
continuous-batching policy (reference ``src/continuous_batch.rs``).

ARB picks each micro-batch from the active sequences by:
* **harmonic length groups** — sequences are grouped (shortest first) so the longest context
  in a group is at most ``harmonic_ratio`` times the shortest; the group with the highest
  summed priority runs (similar lengths keep attention work balanced across the batch);
* **priority** = alpha * utility + beta * urgency + gamma * wait, where utility is the mean
  normalised entropy of the sequence's recent top-1 probabilities (uncertain sequences
  benefit most from compute) and wait is a logistic function of the queueing time;
* **confidence coasting** — a sequence whose top-1 probability stayed above a threshold for
  k steps is deprioritised for ``coast_ms`` and then resumes.

These are scheduling policies (host bookkeeping over sequence ids and token counts); the
engine (``air_rs.runtime.engine``) executes the batches they produce.
"""
from __future__ import annotations

import enum
import math
import time
from collections import deque
from dataclasses import dataclass, field


@dataclass
class ArbConfig:
    max_batch_size: int = 64
    max_context_len: int = 8192
    harmonic_ratio: float = 2.0
    priority_alpha: float = 0.6
    priority_beta: float = 0.3
    priority_gamma: float = 0.1
    confidence_exit_threshold: float = 0.97
    confidence_exit_k: int = 4
    coast_ms: float = 50.0
    prefill_chunk_size: int = 512
    kv_slots: int = 64


class Phase(str, enum.Enum):
    PREFILL = "prefill"
    DECODE = "decode"
    COASTING = "coasting"
    FINISHED = "finished"


@dataclass
class SequenceState:
    id: int
    prompt_tokens: list[int]
    urgency: float = 0.0
    phase: Phase = Phase.PREFILL
    prefilled: int = 0
    generated: int = 0
    arrived: float = field(default_factory=time.monotonic)
    slot: int | None = None
    recent_top1: deque = field(default_factory=lambda: deque(maxlen=16))
    high_conf_streak: int = 0
    utility: float = 0.0
    last_token: int | None = None
    resume_at: float = 0.0

    def __post_init__(self):
        self.urgency = min(1.0, max(0.0, self.urgency))
        self.utility = math.log2(max(1, len(self.prompt_tokens))) / math.log2(8192)

    @property
    def current_len(self) -> int:
        return self.prefilled + self.generated

    def priority(self, cfg: ArbConfig, now: float | None = None) -> float:
        wait = (now if now is not None else time.monotonic()) - self.arrived
        w = 1.0 / (1.0 + math.exp(-0.1 * wait))
        return cfg.priority_alpha * self.utility + cfg.priority_beta * self.urgency + cfg.priority_gamma * w

    def record_decode_step(self, top1: float, cfg: ArbConfig):
        self.generated += 1
        self.recent_top1.append(top1)
        self.high_conf_streak = self.high_conf_streak + 1 if top1 >= cfg.confidence_exit_threshold else 0
        ent = sum(-p * math.log(p) for p in self.recent_top1 if 0 < p < 1) / max(1, len(self.recent_top1))
        self.utility = min(1.0, max(0.0, ent / math.log(2)))

    def should_coast(self, cfg: ArbConfig) -> bool:
        return self.phase == Phase.DECODE and self.high_conf_streak >= cfg.confidence_exit_k


class KvSlotAllocator:
    """O(1) free list of KV slots."""

    def __init__(self, capacity: int):
        self.capacity = capacity
        self._free = list(range(capacity - 1, -1, -1))

    def alloc(self) -> int | None:
        return self._free.pop() if self._free else None

    def free(self, slot: int):
        if slot in self._free or not 0 <= slot < self.capacity:
            raise ValueError(f"bad slot free {slot}")
        self._free.append(slot)

    def available(self) -> int:
        return len(self._free)


@dataclass
class HarmonicGroup:
    ids: list[int]
    min_len: int
    max_len: int

    def can_admit(self, n: int, h: float) -> bool:
        lo, hi = min(self.min_len, n), max(self.max_len, n)
        return lo > 0 and hi / lo <= h

    def admit(self, sid: int, n: int):
        self.ids.append(sid)
        self.min_len, self.max_len = min(self.min_len, n), max(self.max_len, n)


@dataclass
class BatchEntry:
    seq_id: int
    slot: int
    tokens: list[int]
    phase: Phase


class ArbScheduler:
    def __init__(self, cfg: ArbConfig | None = None):
        self.cfg = cfg or ArbConfig()
        self.alloc = KvSlotAllocator(self.cfg.kv_slots)
        self.waiting: list[SequenceState] = []
        self.active: dict[int, SequenceState] = {}
        self._next = 0

    def enqueue(self, prompt_tokens: list[int], urgency: float = 0.0) -> int:
        if not prompt_tokens:
            raise ValueError("empty prompt")
        if len(prompt_tokens) > self.cfg.max_context_len:
            raise ValueError("prompt longer than max_context_len")
        s = SequenceState(self._next, list(prompt_tokens), urgency)
        self._next += 1
        self.waiting.append(s)
        return s.id

    def admit_waiting(self):
        now = time.monotonic()
        self.waiting.sort(key=lambda s: -s.priority(self.cfg, now))
        while self.waiting and self.alloc.available():
            s = self.waiting.pop(0)
            s.slot = self.alloc.alloc()
            self.active[s.id] = s

    def build_micro_batch(self) -> list[BatchEntry] | None:
        now = time.monotonic()
        for s in self.active.values():
            if s.phase == Phase.COASTING and now >= s.resume_at:
                s.phase = Phase.DECODE
        cands = sorted((s for s in self.active.values() if s.phase in (Phase.PREFILL, Phase.DECODE)),
                       key=lambda s: (max(1, s.current_len if s.phase == Phase.DECODE else len(s.prompt_tokens)), s.id))
        if not cands:
            return None
        groups: list[HarmonicGroup] = []
        for s in cands:
            n = max(1, s.current_len if s.phase == Phase.DECODE else len(s.prompt_tokens))
            g = next((g for g in groups if len(g.ids) < self.cfg.max_batch_size
                      and g.can_admit(n, self.cfg.harmonic_ratio)), None)
            if g is None:
                groups.append(HarmonicGroup([s.id], n, n))
            else:
                g.admit(s.id, n)
        best = max(groups, key=lambda g: sum(self.active[i].priority(self.cfg, now) for i in g.ids))
        out = []
        for i in best.ids:
            s = self.active[i]
            if s.phase == Phase.PREFILL:
                end = min(len(s.prompt_tokens), s.prefilled + self.cfg.prefill_chunk_size)
                out.append(BatchEntry(i, s.slot, s.prompt_tokens[s.prefilled:end], Phase.PREFILL))
            else:
                out.append(BatchEntry(i, s.slot, [s.last_token if s.last_token is not None else 0], Phase.DECODE))
        return out

    def commit_results(self, results: list[tuple[int, int, float, bool]]):
        """(seq id, sampled token, top-1 probability, is_eos) per entry of the last batch."""
        for sid, tok, p1, eos in results:
            s = self.active.get(sid)
            if s is None:
                continue
            if eos:
                s.phase = Phase.FINISHED
                self.alloc.free(s.slot)
                del self.active[sid]
                continue
            s.last_token = tok
            if s.phase == Phase.PREFILL:
                s.prefilled = min(len(s.prompt_tokens), s.prefilled + self.cfg.prefill_chunk_size)
                if s.prefilled >= len(s.prompt_tokens):
                    s.phase = Phase.DECODE
            elif s.phase == Phase.DECODE:
                s.record_decode_step(0.0 if p1 != p1 else p1, self.cfg)
                if s.should_coast(self.cfg):
                    s.phase = Phase.COASTING
                    s.resume_at = time.monotonic() + self.cfg.coast_ms / 1e3
                    s.high_conf_streak = 0


# ---------------------------------------------------------------------------- Orca / Sarathi
class Priority(enum.IntEnum):
    LOW = 0
    NORMAL = 1
    HIGH = 2
    CRITICAL = 3


@dataclass
class ManagedRequest:
    id: int
    prompt_len: int
    max_tokens: int
    priority: Priority = Priority.NORMAL
    prefilled: int = 0
    generated: int = 0
    arrived: float = field(default_factory=time.monotonic)

    @property
    def in_prefill(self) -> bool:
        return self.prefilled < self.prompt_len

    @property
    def done(self) -> bool:
        return self.generated >= self.max_tokens


@dataclass
class ScheduledBatch:
    decode: list[int]                       # request ids decoding one token
    prefill: list[tuple[int, int, int]]     # (request id, start, n tokens)

    @property
    def num_tokens(self) -> int:
        return len(self.decode) + sum(n for _, _, n in self.prefill)


class ContinuousBatchScheduler:
    """Iteration-level scheduling with a per-step token budget: every running request
    decodes one token, and the rest of the budget goes to prompt chunks, highest priority
    (then oldest) first (Orca iteration scheduling + Sarathi chunked prefill)."""

    def __init__(self, max_batch: int = 64, token_budget: int = 2048, chunk: int = 512):
        self.max_batch, self.budget, self.chunk = max_batch, token_budget, chunk
        self.requests: dict[int, ManagedRequest] = {}
        self._next = 0

    def submit(self, prompt_len: int, max_tokens: int, priority: Priority = Priority.NORMAL) -> int:
        rid = self._next
        self._next += 1
        self.requests[rid] = ManagedRequest(rid, prompt_len, max_tokens, priority)
        return rid

    def abort(self, rid: int) -> bool:
        return self.requests.pop(rid, None) is not None

    def schedule(self) -> ScheduledBatch:
        running = [r for r in self.requests.values() if not r.in_prefill and not r.done]
        decode = [r.id for r in sorted(running, key=lambda r: (-r.priority, r.arrived))][: self.max_batch]
        left = self.budget - len(decode)
        slots = self.max_batch - len(decode)
        prefill = []
        for r in sorted((r for r in self.requests.values() if r.in_prefill), key=lambda r: (-r.priority, r.arrived)):
            if left <= 0 or slots <= 0:
                break
            n = min(self.chunk, r.prompt_len - r.prefilled, left)
            prefill.append((r.id, r.prefilled, n))
            left -= n
            slots -= 1
        return ScheduledBatch(decode, prefill)

    def prefill_done(self, rid: int, n: int):
        r = self.requests[rid]
        r.prefilled += n
        if not r.in_prefill:
            r.generated += 1            # the chunk that completes the prompt samples a token

    def decode_step(self, rids: list[int]) -> list[int]:
        """Advance the decoded requests; returns the ids that finished (and removes them)."""
        out = []
        for rid in rids:
            r = self.requests[rid]
            r.generated += 1
            if r.done:
                out.append(rid)
                del self.requests[rid]
        return out
