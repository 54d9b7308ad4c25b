"""Neuron-predicate FFN loading (reference ``src/neuron_predicate.rs``: NeuronMask rounded to
64-neuron bundles, BundleMap coalescing active bundles into contiguous reads, NeuronPredictor =
ReLU(h W_down + b) W_up -> sigmoid scores > threshold, predicate cache across tokens).

Applied to layer streaming: only the bundles of FFN rows (gate / up rows, down columns)
a token is predicted to use need to be copied host -> HBM; ``sparse_ffn`` computes the FFN
over just those rows, which is what the loaded subset can produce, so the accuracy cost of a
predictor can be measured against the dense FFN.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

BUNDLE_SIZE = 64
PREDICTOR_RATIO = 8
DEFAULT_ACTIVATION_THRESHOLD = 0.5
MIN_USEFUL_SPARSITY = 0.30
FFN_WEIGHT_FRACTION = 0.663


class NeuronMask:
    def __init__(self, active: torch.Tensor):
        """``active`` bool [d_ffn]; rounded up to whole bundles."""
        d = active.numel()
        nb = (d + BUNDLE_SIZE - 1) // BUNDLE_SIZE
        padded = F.pad(active.bool(), (0, nb * BUNDLE_SIZE - d))
        self.bundles = padded.reshape(nb, BUNDLE_SIZE).any(-1)
        self.d_ffn = d

    @classmethod
    def all_active(cls, d: int) -> "NeuronMask":
        return cls(torch.ones(d, dtype=torch.bool))

    @classmethod
    def all_inactive(cls, d: int) -> "NeuronMask":
        return cls(torch.zeros(d, dtype=torch.bool))

    @classmethod
    def from_scores(cls, scores: torch.Tensor, threshold: float = DEFAULT_ACTIVATION_THRESHOLD) -> "NeuronMask":
        return cls(scores >= threshold)

    @classmethod
    def from_bundles(cls, active_bundles, d: int) -> "NeuronMask":
        b = torch.as_tensor(active_bundles, dtype=torch.bool)
        return cls(b.repeat_interleave(BUNDLE_SIZE)[:d])

    def neurons(self) -> torch.Tensor:
        return self.bundles.repeat_interleave(BUNDLE_SIZE)[: self.d_ffn]

    def is_active(self, i: int) -> bool:
        return bool(self.bundles[i // BUNDLE_SIZE])

    def n_bundles(self) -> int:
        return self.bundles.numel()

    def active_bundles(self) -> int:
        return int(self.bundles.sum())

    def active_count(self) -> int:
        return int(self.neurons().sum())

    def sparsity(self) -> float:
        return 1.0 - self.active_count() / max(1, self.d_ffn)

    def bandwidth_saving(self) -> float:
        """Fraction of a layer's bytes not read (FFN share of the layer x sparsity)."""
        return FFN_WEIGHT_FRACTION * self.sparsity()


@dataclass
class BundleRange:
    start_bundle: int
    end_bundle: int

    def __len__(self):
        return self.end_bundle - self.start_bundle

    def byte_offset(self, bytes_per_neuron: int) -> int:
        return self.start_bundle * BUNDLE_SIZE * bytes_per_neuron

    def byte_len(self, bytes_per_neuron: int) -> int:
        return len(self) * BUNDLE_SIZE * bytes_per_neuron


class BundleMap:
    def __init__(self, mask: NeuronMask):
        self.ranges: list[BundleRange] = []
        b = mask.bundles.tolist()
        i = 0
        while i < len(b):
            if b[i]:
                s = i
                while i < len(b) and b[i]:
                    i += 1
                self.ranges.append(BundleRange(s, i))
            else:
                i += 1
        self.total_bundles = sum(len(r) for r in self.ranges)
        self.total_neurons = self.total_bundles * BUNDLE_SIZE

    def n_reads(self) -> int:
        return len(self.ranges)

    def total_bytes(self, bytes_per_neuron: int) -> int:
        return self.total_neurons * bytes_per_neuron

    def io_ranges(self, bytes_per_neuron: int) -> list[tuple[int, int]]:
        return [(r.byte_offset(bytes_per_neuron), r.byte_len(bytes_per_neuron)) for r in self.ranges]


class NeuronPredictor:
    def __init__(self, w_down: torch.Tensor, w_up: torch.Tensor, b_down: torch.Tensor | None = None,
                 threshold: float = DEFAULT_ACTIVATION_THRESHOLD):
        """w_down [hidden, d/8], w_up [d/8, d]."""
        self.w_down, self.w_up, self.b_down, self.threshold = w_down, w_up, b_down, threshold

    @classmethod
    def random(cls, hidden: int, d_ffn: int, seed: int = 0, threshold: float = DEFAULT_ACTIVATION_THRESHOLD):
        g = torch.Generator().manual_seed(seed)
        p = d_ffn // PREDICTOR_RATIO
        wd = (torch.rand(hidden, p, generator=g) * 2 - 1) * (2.0 / (hidden + p)) ** 0.5
        wu = (torch.rand(p, d_ffn, generator=g) * 2 - 1) * (2.0 / (p + d_ffn)) ** 0.5
        return cls(wd, wu, None, threshold)

    def scores(self, h: torch.Tensor) -> torch.Tensor:
        mid = h.float() @ self.w_down
        if self.b_down is not None:
            mid = mid + self.b_down
        return torch.sigmoid(torch.relu(mid) @ self.w_up)

    def predict(self, h: torch.Tensor) -> NeuronMask:
        """Union over the rows of ``h`` (a batch loads what any of its tokens needs)."""
        s = self.scores(h.reshape(-1, h.shape[-1]))
        return NeuronMask.from_scores(s.amax(0), self.threshold)


class PredicateCache:
    """Reuse a layer's mask while consecutive hidden states stay close (cosine >= tau)."""

    def __init__(self, tau: float = 0.95):
        self.tau = tau
        self._last: dict[int, tuple[torch.Tensor, NeuronMask]] = {}
        self.hits = self.misses = 0

    def get(self, layer: int, h: torch.Tensor, predictor: NeuronPredictor) -> NeuronMask:
        prev = self._last.get(layer)
        v = h.reshape(-1).float()
        if prev is not None and float(F.cosine_similarity(prev[0], v, dim=0)) >= self.tau:
            self.hits += 1
            return prev[1]
        self.misses += 1
        m = predictor.predict(h)
        self._last[layer] = (v, m)
        return m


def sparse_ffn(x: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor,
               mask: NeuronMask) -> torch.Tensor:
    """SwiGLU FFN over the active neurons only (the rows a predicated load brings in)."""
    idx = mask.neurons().nonzero().flatten().to(x.device)
    g = x.float() @ w_gate[idx].float().t()
    u = x.float() @ w_up[idx].float().t()
    return (F.silu(g) * u) @ w_down[:, idx].float().t()
