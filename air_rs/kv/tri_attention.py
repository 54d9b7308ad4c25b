"""TriAttention token-importance scoring for KV eviction (reference ``src/tri_attention.rs``).

For each cached position i (reference ``src/tri_attention.rs:17-28, 93-129``):

    sim_i   = mean over heads of clamp(q_agg,h . k_i,h * d^-1/4 / (|q_agg,h| |k_i,h|), -1, 1)
    phase_i = (mean over RoPE frequencies theta_j of cos(theta_j * i) + 1) / 2
    score_i = clamp(alpha * sim_i + (1 - alpha) * phase_i, 0, 1)

with alpha = 0.7; the first ``SINK_COUNT`` = 4 positions (attention sinks) score 1 and are
always kept, and the other scores are min-max normalised. ``q_agg`` is the mean query over a
recent observation window (SnapKV-style). Here the whole sequence is scored in one batched
tensor expression (works on CPU or on the GPU against the paged pool's keys) instead of a
per-position loop, and ``keep_mask`` returns the top-``budget`` positions.

``TriAttentionTierManager`` plugs the score into the HERMES tier manager: positions are
demoted in increasing TriAttention score instead of the recency/density score.
"""
from __future__ import annotations

import torch

from .tiers import HermesTierManager

SINK_COUNT = 4
ALPHA = 0.7
MIN_BUDGET = SINK_COUNT + 1


class TriScorer:
    def __init__(self, head_dim: int, n_heads: int, rope_base: float):
        if head_dim <= 0 or head_dim % 2:
            raise ValueError("head_dim must be even and positive")
        if n_heads <= 0:
            raise ValueError("n_heads must be positive")
        self.head_dim, self.n_heads = head_dim, n_heads
        self.rope_freqs = 1.0 / rope_base ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim)
        self.scale = head_dim ** -0.25

    def phase(self, positions: torch.Tensor) -> torch.Tensor:
        f = self.rope_freqs.to(positions.device)
        return (torch.cos(positions.float()[:, None] * f[None]).mean(-1) + 1.0) * 0.5

    def score(self, q_agg: torch.Tensor, k_cache: torch.Tensor) -> torch.Tensor:
        """q_agg [n_heads * head_dim] (or [n_heads, head_dim]); k_cache [seq, n_heads, head_dim]
        (or flat [seq, n_heads * head_dim]). Returns scores [seq] in [0, 1]."""
        H, D = self.n_heads, self.head_dim
        q = q_agg.float().reshape(H, D)
        k = k_cache.float().reshape(-1, H, D)
        S = k.shape[0]
        dot = (k * q[None]).sum(-1)                                   # [S, H]
        den = k.norm(dim=-1) * q.norm(dim=-1)[None]
        cos = torch.where(den < 1e-8, torch.zeros_like(dot), (dot * self.scale / den.clamp_min(1e-30)).clamp(-1, 1))
        sim = cos.mean(-1)
        pos = torch.arange(S, device=k.device)
        raw = (ALPHA * sim + (1.0 - ALPHA) * self.phase(pos)).clamp(0.0, 1.0)
        raw[:SINK_COUNT] = 1.0
        if S > SINK_COUNT:
            rest = raw[SINK_COUNT:]
            lo, hi = rest.min(), rest.max()
            if float(hi - lo) >= 1e-8:
                raw[SINK_COUNT:] = (rest - lo) / (hi - lo)
        return raw

    @staticmethod
    def keep_mask(scores: torch.Tensor, budget: int) -> torch.Tensor:
        """True = retain: the ``budget`` (at least MIN_BUDGET) highest scores, sinks first on ties."""
        n = scores.numel()
        budget = min(max(budget, MIN_BUDGET), n)
        # stable order: higher score first, then lower position (sinks win ties at 1.0)
        order = sorted(range(n), key=lambda i: (-float(scores[i]), i))
        mask = torch.zeros(n, dtype=torch.bool)
        mask[order[:budget]] = True
        return mask


def observation_query(q_window: torch.Tensor) -> torch.Tensor:
    """Mean query over a recent window [W, n_heads, head_dim] -> [n_heads * head_dim]."""
    return q_window.float().mean(0).reshape(-1)


class TriAttentionTierManager(HermesTierManager):
    """HERMES tier manager variant ordering demotions by TriAttention score.

    ``update_scores(q_agg, k_cache)`` rescores the tracked positions; ``enforce_budgets``
    demotes the lowest-scoring (non-pinned) positions first, ties broken by position."""

    def __init__(self, budget=None, scorer: TriScorer | None = None):
        super().__init__(budget)
        self.scorer = scorer
        self.tri_scores: dict[int, float] = {}

    def update_scores(self, q_agg: torch.Tensor, k_cache: torch.Tensor):
        s = self.scorer.score(q_agg, k_cache)
        self.tri_scores = {i: float(v) for i, v in enumerate(s.tolist())}

    def enforce_budgets(self):
        sc = self.tri_scores
        self._enforce(lambda tier: sorted((e for e in self.entries.values() if e.tier == tier),
                                          key=lambda e: (sc.get(e.position, 0.0), e.position)))
