"""LoRA / QLoRA adapters (reference ``src/lora.rs``, ``src/qlora.rs``): an LRU adapter cache,
a multi-adapter pool keyed by request, and the low-rank update W' = W + (alpha / r) * B @ A.

Adapters are applied by merging into a dense (bf16) copy of the target weight
(``merge_into``) or as a side path on activations (``LoraAdapter.delta``: x @ A^T @ B^T
scaled), which is how a quantised base weight (QLoRA) keeps its blocks untouched.
"""
from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass, field

import torch


@dataclass
class LoraAdapter:
    name: str
    # target weight name -> (A [r, K], B [N, r])
    layers: dict[str, tuple[torch.Tensor, torch.Tensor]] = field(default_factory=dict)
    alpha: float = 16.0

    @property
    def rank(self) -> int:
        return next(iter(self.layers.values()))[0].shape[0] if self.layers else 0

    @property
    def scale(self) -> float:
        return self.alpha / max(1, self.rank)

    def delta(self, target: str, x: torch.Tensor) -> torch.Tensor:
        """(alpha/r) * x @ A^T @ B^T for activations x [T, K]."""
        a, b = self.layers[target]
        return (x.to(a.dtype) @ a.t() @ b.t()) * self.scale

    def merge_into(self, target: str, w: torch.Tensor) -> torch.Tensor:
        """W + (alpha/r) * B @ A (w: dense [N, K]); returns a new tensor."""
        a, b = self.layers[target]
        return (w.float() + self.scale * (b.float() @ a.float())).to(w.dtype)

    def nbytes(self) -> int:
        return sum(a.numel() * a.element_size() + b.numel() * b.element_size() for a, b in self.layers.values())

    @classmethod
    def random(cls, name: str, shapes: dict[str, tuple[int, int]], rank: int = 8, alpha: float = 16.0,
               seed: int = 0, dtype=torch.float32) -> "LoraAdapter":
        g = torch.Generator().manual_seed(seed)
        layers = {t: ((torch.randn(rank, k, generator=g) * 0.01).to(dtype),
                      (torch.randn(n, rank, generator=g) * 0.01).to(dtype)) for t, (n, k) in shapes.items()}
        return cls(name, layers, alpha)


class AdapterCache:
    """LRU cache of loaded adapters bounded by count and bytes."""

    def __init__(self, max_adapters: int = 8, max_bytes: int | None = None, loader=None):
        self.max_adapters, self.max_bytes, self.loader = max_adapters, max_bytes, loader
        self._d: OrderedDict[str, LoraAdapter] = OrderedDict()
        self.hits = self.misses = self.evictions = 0

    def _bytes(self) -> int:
        return sum(a.nbytes() for a in self._d.values())

    def put(self, adapter: LoraAdapter):
        self._d[adapter.name] = adapter
        self._d.move_to_end(adapter.name)
        while len(self._d) > self.max_adapters or (self.max_bytes is not None and self._bytes() > self.max_bytes
                                                   and len(self._d) > 1):
            self._d.popitem(last=False)
            self.evictions += 1

    def get(self, name: str) -> LoraAdapter | None:
        a = self._d.get(name)
        if a is not None:
            self.hits += 1
            self._d.move_to_end(name)
            return a
        self.misses += 1
        if self.loader is not None:
            a = self.loader(name)
            if a is not None:
                self.put(a)
        return a

    def __contains__(self, name):
        return name in self._d

    def __len__(self):
        return len(self._d)


class MultiLoraPool:
    """Per-request adapter selection over a shared cache (requests without one use the base)."""

    def __init__(self, cache: AdapterCache):
        self.cache = cache
        self.assignments: dict[int, str] = {}

    def assign(self, request_id: int, adapter: str | None):
        if adapter is None:
            self.assignments.pop(request_id, None)
        else:
            self.assignments[request_id] = adapter

    def apply(self, request_ids: list[int], target: str, x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
        """y[i] += delta of request i's adapter (rows grouped by adapter)."""
        groups: dict[str, list[int]] = {}
        for i, rid in enumerate(request_ids):
            name = self.assignments.get(rid)
            if name is not None:
                groups.setdefault(name, []).append(i)
        for name, rows in groups.items():
            ad = self.cache.get(name)
            if ad is None or target not in ad.layers:
                continue
            idx = torch.tensor(rows, device=x.device)
            y.index_add_(0, idx, ad.delta(target, x.index_select(0, idx)).to(y.dtype))
        return y


@dataclass
class QLoraAdapter:
    """Low-rank update over a quantised base weight: y = dequant(W) x + (alpha/r) B A x."""
    base: object                      # ops.QWeight or a dense tensor
    adapter: LoraAdapter
    target: str

    def forward_reference(self, x: torch.Tensor) -> torch.Tensor:
        from . import ops
        w = self.base.dequantize_bf16().float() if isinstance(self.base, ops.QWeight) else self.base.float()
        return x.float() @ w.t() + self.adapter.delta(self.target, x.float())
