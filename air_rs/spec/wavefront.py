"""Wavefront decoding policy: FFN activation-sparsity prediction, the union of the active
neurons of a draft wavefront, adaptive draft size, and per-cycle accounting (reference
``src/wavefront.rs`` WavefrontConfig / CycleStats / WavefrontSession / compute_union_mask /
WavefrontHealthMonitor, and ``src/sparsity_predictor.rs`` SparsityConfig /
LayerSparsityPredictor / SparsityPredictorBank / SparseWeightMask).

A cycle drafts K tokens (Medusa heads), predicts for each drafted position which FFN
neurons of each layer will be active, and needs only the union of those rows of gate/up
(and columns of down) to verify the K drafts in one batch. On a B200 that keeps every layer
in HBM this saves nothing; it pays where layers stream from host memory (only the active
rows need to cross PCIe) and is reported per cycle as ``bytes_saved``.

The predictor is a per-layer logistic model ``sigmoid(W h)`` over the FFN input ``h`` whose
top ``ceil(I * fraction)`` scores are the predicted active neurons; it trains online by SGD
on the observed gates (a neuron is active when ``|silu(gate) * up| > threshold``). All of it
is batched torch on the tensors' device: predictions for a whole wavefront are one
[K, H] x [H, I] product and one ``topk``. ``SparseFFNHook`` attaches a bank to the CPU oracle
model's FFN (``OracleModel.ffn_hook``) to train it on real activations and, when masking,
to zero the neurons outside the predicted set — the numerics of computing only those rows.
"""
from __future__ import annotations

import math
from collections import deque
from dataclasses import dataclass, field

import torch

ACTIVE_THRESHOLD = 0.1


# ---------------------------------------------------------------------------- predictor
@dataclass
class SparsityConfig:
    hidden_dim: int
    intermediate_dim: int
    top_k_fraction: float = 0.2

    @classmethod
    def for_model(cls, hidden_dim: int, intermediate_dim: int) -> "SparsityConfig":
        return cls(hidden_dim, intermediate_dim, 0.2)

    def top_k(self) -> int:
        return min(self.intermediate_dim, max(1, math.ceil(self.intermediate_dim * self.top_k_fraction)))


@dataclass
class SparseWeightMask:
    """Sorted active row indices of an [I, H] FFN weight (gate/up rows, down columns)."""
    active_indices: torch.Tensor          # int64, sorted, unique
    total_rows: int

    @classmethod
    def dense(cls, total_rows: int) -> "SparseWeightMask":
        return cls(torch.arange(total_rows), total_rows)

    def n_active(self) -> int:
        return int(self.active_indices.numel())

    def density(self) -> float:
        return self.n_active() / self.total_rows if self.total_rows else 1.0

    def bytes_saved(self, col_dim: int, bytes_per_weight: float = 2.0, n_matrices: int = 3) -> int:
        """Bytes not moved for the inactive rows of ``n_matrices`` [I, col_dim] weights."""
        return int((self.total_rows - self.n_active()) * col_dim * bytes_per_weight * n_matrices)

    def as_bool(self, device=None) -> torch.Tensor:
        m = torch.zeros(self.total_rows, dtype=torch.bool, device=device)
        m[self.active_indices.to(m.device)] = True
        return m


class LayerSparsityPredictor:
    def __init__(self, config: SparsityConfig, weight: torch.Tensor | None = None, seed: int = 0,
                 device="cpu"):
        self.config = config
        if weight is None:
            g = torch.Generator().manual_seed(seed)
            scale = math.sqrt(2.0 / config.hidden_dim)
            weight = (torch.rand(config.intermediate_dim, config.hidden_dim, generator=g) * 2 - 1) * scale
        self.w = weight.float().to(device)
        self.accuracy_ema = 0.5

    @classmethod
    def zeros(cls, config: SparsityConfig, device="cpu") -> "LayerSparsityPredictor":
        p = cls(config, torch.zeros(config.intermediate_dim, config.hidden_dim), device=device)
        p.accuracy_ema = 0.0
        return p

    def scores(self, hidden: torch.Tensor) -> torch.Tensor:
        """[..., H] -> [..., I] activation probabilities."""
        return torch.sigmoid(hidden.float().to(self.w.device) @ self.w.t())

    def predict_active(self, hidden: torch.Tensor) -> torch.Tensor:
        """[H] -> sorted [k] indices; [B, H] -> [B, k] (each row sorted)."""
        idx = torch.topk(self.scores(hidden), self.config.top_k(), dim=-1).indices
        return idx.sort(dim=-1).values

    def update(self, hidden: torch.Tensor, actual: torch.Tensor, lr: float = 1e-4,
               threshold: float = ACTIVE_THRESHOLD):
        """One logistic-regression SGD step per row of ``hidden`` [B, H] against the observed
        activations ``actual`` [B, I] (active = |a| > threshold), summed over the batch."""
        h = hidden.float().reshape(-1, self.config.hidden_dim).to(self.w.device)
        t = (actual.float().reshape(h.shape[0], -1).abs() > threshold).float().to(self.w.device)
        grad = torch.sigmoid(h @ self.w.t()) - t                  # [B, I]
        self.w -= lr * grad.t() @ h

    def measure_accuracy(self, predicted: torch.Tensor, actual: torch.Tensor,
                         threshold: float = ACTIVE_THRESHOLD) -> float:
        """Recall of the truly active neurons by the predicted sets, row by row for a batch
        ([B, k] predicted, [B, I] actual; 1.0 with none active); folded into ``accuracy_ema``
        with weight 0.1."""
        I = self.config.intermediate_dim
        act = actual.float().reshape(-1, I).abs() > threshold             # [B, I]
        n = int(act.sum())
        if n == 0:
            return 1.0
        hit = torch.zeros_like(act)
        hit.scatter_(1, predicted.reshape(act.shape[0], -1).to(act.device), True)
        acc = float((act & hit).sum()) / n
        self.accuracy_ema = 0.9 * self.accuracy_ema + 0.1 * acc
        return acc


class SparsityPredictorBank:
    def __init__(self, n_layers: int, config: SparsityConfig, seed: int = 0, device="cpu"):
        self.config = config
        self.predictors = [LayerSparsityPredictor(config, seed=seed + i, device=device) for i in range(n_layers)]

    def predict(self, layer_id: int, hidden: torch.Tensor) -> torch.Tensor:
        return self.predictors[layer_id].predict_active(hidden)

    def predict_mask(self, hidden: torch.Tensor, layer_id: int) -> SparseWeightMask:
        """Mask for one position, or the union over the rows of a [K, H] wavefront."""
        idx = self.predict(layer_id, hidden)
        if idx.dim() == 1:
            return SparseWeightMask(idx.cpu(), self.config.intermediate_dim)
        return compute_union_mask(list(idx.cpu()), self.config.intermediate_dim)

    def update(self, layer_id: int, hidden: torch.Tensor, actual: torch.Tensor, lr: float = 1e-4):
        self.predictors[layer_id].update(hidden, actual, lr)

    def mean_accuracy(self) -> float:
        return sum(p.accuracy_ema for p in self.predictors) / max(1, len(self.predictors))

    def bandwidth_reduction(self) -> float:
        return 1.0 / self.config.top_k_fraction


def compute_union_mask(per_token_indices: list, total_rows: int) -> SparseWeightMask:
    """Union of the active rows of every drafted position; dense when there are none.
    Indices outside [0, total_rows) are ignored."""
    if not per_token_indices:
        return SparseWeightMask.dense(total_rows)
    m = torch.zeros(total_rows, dtype=torch.bool)
    for ix in per_token_indices:
        ix = torch.as_tensor(ix, dtype=torch.long).reshape(-1)
        ix = ix[(ix >= 0) & (ix < total_rows)]
        m[ix] = True
    return SparseWeightMask(m.nonzero().reshape(-1), total_rows)


# ---------------------------------------------------------------------------- oracle hook
class SparseFFNHook:
    """``OracleModel.ffn_hook``: sees every FFN activation ``a = silu(g) * u`` [S, I] with its
    input ``h`` [S, H]. ``learn`` trains the layer's predictor on it; ``mask`` zeroes the
    neurons outside the union of the predicted sets of the S positions (what computing only
    those rows gives). Keeps per-layer recall and the density of the masks applied."""

    def __init__(self, bank: SparsityPredictorBank, learn: bool = True, mask: bool = False, lr: float = 1e-3):
        self.bank, self.learn, self.mask, self.lr = bank, learn, mask, lr
        self.densities: list[float] = []
        self.recalls: list[float] = []

    def __call__(self, layer: int, h: torch.Tensor, a: torch.Tensor) -> torch.Tensor:
        p = self.bank.predictors[layer]
        idx = p.predict_active(h)
        self.recalls.append(p.measure_accuracy(idx, a))
        if self.learn:
            p.update(h, a, self.lr)
        if not self.mask:
            return a
        m = compute_union_mask(list(idx.reshape(h.shape[0], -1)), a.shape[-1])
        self.densities.append(m.density())
        return a * m.as_bool(a.device).to(a.dtype)


# ---------------------------------------------------------------------------- wavefront loop
@dataclass
class WavefrontConfig:
    draft_size: int = 8
    sparsity_fraction: float = 0.15
    async_double_buffer: bool = True
    min_acceptance_rate: float = 0.4
    verbose: bool = True

    @classmethod
    def disabled(cls) -> "WavefrontConfig":
        return cls(draft_size=1, async_double_buffer=False)

    @classmethod
    def aggressive(cls, draft_size: int) -> "WavefrontConfig":
        return cls(draft_size, 0.20, True, 0.4, False)


@dataclass
class CycleStats:
    draft_ms: float = 0.0
    io_ms: float = 0.0
    verify_ms: float = 0.0
    tokens_accepted: int = 0
    tokens_drafted: int = 0
    sparsity_density: float = 1.0
    bytes_saved: int = 0

    def total_ms(self) -> float:
        return self.draft_ms + self.io_ms + self.verify_ms

    def effective_tps(self) -> float:
        t = self.total_ms()
        return self.tokens_accepted / (t / 1000.0) if t > 0 else 0.0

    def display(self) -> str:
        return (f"draft={self.draft_ms:.1f}ms | io={self.io_ms:.1f}ms | verify={self.verify_ms:.1f}ms | "
                f"accept={self.tokens_accepted}/{self.tokens_drafted} | density={self.sparsity_density * 100:.0f}% | "
                f"saved={self.bytes_saved / 1e6:.1f}MB | {self.effective_tps():.2f} tok/s")


@dataclass
class WavefrontSession:
    total_tokens: int = 0
    total_cycles: int = 0
    total_bytes_saved: int = 0
    total_wall_ms: float = 0.0
    drafted: int = 0
    accepted: int = 0

    def record(self, c: CycleStats):
        """A cycle yields its accepted drafts plus the target's own next token."""
        self.drafted += c.tokens_drafted
        self.accepted += c.tokens_accepted
        self.total_tokens += c.tokens_accepted + 1
        self.total_cycles += 1
        self.total_bytes_saved += c.bytes_saved
        self.total_wall_ms += c.total_ms()

    def acceptance_rate(self) -> float:
        return self.accepted / self.drafted if self.drafted else 0.0

    def speedup_estimate(self) -> float:
        """Tokens per cycle over the one token a plain decode step yields."""
        return self.total_tokens / self.total_cycles if self.total_cycles else 1.0

    def overall_tps(self) -> float:
        return self.total_tokens / (self.total_wall_ms / 1000.0) if self.total_wall_ms > 0 else 0.0

    def summary(self) -> str:
        return (f"wavefront: {self.total_tokens} tokens in {self.total_cycles} cycles, "
                f"{self.total_wall_ms / 1000.0:.2f} s, {self.overall_tps():.2f} tok/s, "
                f"{self.speedup_estimate():.2f} tokens/cycle, acceptance {self.acceptance_rate() * 100:.1f}%, "
                f"{self.total_bytes_saved / 1e9:.2f} GB not streamed")


@dataclass
class WavefrontHealthMonitor:
    """Acceptance rates of the last ``window_size`` cycles; from five cycles on, a mean above
    0.85 grows the draft by 2 and a mean below 0.50 halves it (within [min, max])."""
    current_draft_size: int = 8
    window_size: int = 20
    min_draft_size: int = 1
    max_draft_size: int = 64
    window: deque = field(default_factory=deque)

    def update(self, accepted: int, drafted: int):
        if drafted <= 0:
            return
        self.window.append(accepted / drafted)
        while len(self.window) > self.window_size:
            self.window.popleft()
        if len(self.window) >= 5:
            mean = self.mean_acceptance()
            if mean > 0.85:
                self.current_draft_size = min(self.current_draft_size + 2, self.max_draft_size)
            if mean < 0.50:
                self.current_draft_size = max(self.current_draft_size // 2, self.min_draft_size)

    def mean_acceptance(self) -> float:
        return sum(self.window) / len(self.window) if self.window else 0.0
