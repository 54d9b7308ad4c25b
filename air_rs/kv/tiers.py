"""KV tier policy (reference ``src/kv_tier.rs``): per-position tier metadata — Pinned and
Active in HBM, Warm in host RAM, Cold on disk — with budgets, LRU demotion, promotion on
access, and the HERMES importance score (recency, access density, prefix position).

This module is the policy; the data movement for the Warm tier is ``KvSwapManager`` (whole
sequences, pinned host memory) and for the Cold tier ``save_cold``/``load_cold`` (KV blocks
to a file and back).
"""
from __future__ import annotations

import enum
import math
import time
from dataclasses import dataclass, field

import torch


class KvTier(str, enum.Enum):
    PINNED = "pinned"
    ACTIVE = "active"
    WARM = "warm"
    COLD = "cold"


@dataclass
class TokenEntry:
    position: int
    tier: KvTier
    access_count: int = 0
    last_access: float = field(default_factory=time.monotonic)
    last_step: int = 0

    @property
    def is_pinned(self) -> bool:
        return self.tier == KvTier.PINNED

    def touch(self, step: int = 0):
        self.access_count += 1
        self.last_access = time.monotonic()
        self.last_step = step


@dataclass
class TierBudget:
    pinned_max: int = 512
    active_max: int = 2048
    warm_max: int = 8192

    @classmethod
    def from_vram(cls, vram_bytes: int, bytes_per_token: int) -> "TierBudget":
        """20 % of the HBM token capacity pinned, the rest active; host RAM holds 4x active."""
        if bytes_per_token <= 0:
            return cls()
        tokens = vram_bytes // bytes_per_token
        pinned = tokens * 20 // 100
        active = tokens - pinned
        return cls(max(pinned, 64), max(active, 256), active * 4)


class TierManager:
    def __init__(self, budget: TierBudget | None = None):
        self.budget = budget or TierBudget()
        self.entries: dict[int, TokenEntry] = {}
        self.step = 0

    def add_token(self, position: int):
        self.entries[position] = TokenEntry(position, KvTier.ACTIVE, last_step=self.step)
        self.step += 1

    def pin_range(self, start: int, end: int):
        for p in range(start, end):
            e = self.entries.get(p)
            if e is None:
                e = self.entries[p] = TokenEntry(p, KvTier.PINNED)
            if sum(1 for x in self.entries.values() if x.tier == KvTier.PINNED) < self.budget.pinned_max \
                    or e.tier == KvTier.PINNED:
                e.tier = KvTier.PINNED

    def touch_positions(self, positions):
        for p in positions:
            e = self.entries.get(p)
            if e is not None:
                e.touch(self.step)

    def get_tier(self, position: int) -> KvTier | None:
        e = self.entries.get(position)
        return e.tier if e is not None else None

    def _demotion_order(self, tier: KvTier) -> list[TokenEntry]:
        """Least recently used first."""
        return sorted((e for e in self.entries.values() if e.tier == tier), key=lambda e: (e.last_step, e.position))

    def enforce_budgets(self):
        self._enforce(self._demotion_order)

    def _enforce(self, order):
        act = order(KvTier.ACTIVE)
        for e in act[:max(0, len(act) - self.budget.active_max)]:
            e.tier = KvTier.WARM
        warm = order(KvTier.WARM)
        for e in warm[:max(0, len(warm) - self.budget.warm_max)]:
            e.tier = KvTier.COLD

    def promote(self, position: int) -> bool:
        """Bring a Warm/Cold position back to Active (on access); False if already in HBM."""
        e = self.entries.get(position)
        if e is None or e.tier in (KvTier.PINNED, KvTier.ACTIVE):
            return False
        e.tier = KvTier.ACTIVE
        e.touch(self.step)
        return True

    def count_tier(self, tier: KvTier) -> int:
        return sum(1 for e in self.entries.values() if e.tier == tier)

    def total_positions(self) -> int:
        return len(self.entries)

    def distribution(self) -> tuple[int, int, int, int]:
        return tuple(self.count_tier(t) for t in (KvTier.PINNED, KvTier.ACTIVE, KvTier.WARM, KvTier.COLD))

    def clear(self):
        self.entries.clear()

    def summary(self) -> str:
        p, a, w, c = self.distribution()
        return f"KV tiers: pinned={p} active={a} warm={w} cold={c}"


@dataclass
class HermesWeights:
    alpha: float = 0.40
    beta: float = 0.35
    gamma: float = 0.25
    lam: float = 0.05
    sigma: float = 0.1
    prefix_len: int = 128

    def score(self, e: TokenEntry, current_step: int) -> float:
        """alpha*recency + beta*access density + gamma*prefix-position weight."""
        recency = math.exp(-self.lam * max(0, current_step - e.last_step))
        density = min(1.0, math.log(1.0 + e.access_count) / math.log(10.0))
        pos_w = 1.0 / (1.0 + math.exp(-self.sigma * (self.prefix_len - e.position)))
        return self.alpha * recency + self.beta * density + self.gamma * pos_w


class HermesTierManager(TierManager):
    """Demotes the lowest-HERMES-score positions first instead of the least recently used."""

    def __init__(self, budget: TierBudget | None = None, weights: HermesWeights | None = None):
        super().__init__(budget)
        self.weights = weights or HermesWeights()

    def enforce_budgets_hermes(self):
        step = self.step
        self._enforce(lambda tier: sorted((e for e in self.entries.values() if e.tier == tier),
                                          key=lambda e: (self.weights.score(e, step), e.position)))

    enforce_budgets = enforce_budgets_hermes


def save_cold(path: str, kv: torch.Tensor, blocks: list[int]):
    """Cold tier: write the listed KV blocks of every layer to ``path``."""
    idx = torch.tensor(blocks, dtype=torch.long, device=kv.device)
    torch.save({"blocks": blocks, "kv": kv.index_select(1, idx).cpu()}, path)


def load_cold(path: str, kv: torch.Tensor, blocks: list[int]):
    """Load blocks saved by ``save_cold`` into (possibly different) block ids ``blocks``."""
    d = torch.load(path)
    idx = torch.tensor(blocks, dtype=torch.long, device=kv.device)
    kv.index_copy_(1, idx, d["kv"].to(kv.device))
