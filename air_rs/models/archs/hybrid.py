"""Per-layer attention backends (reference ``src/attention_backend.rs``: AttentionBackend,
HybridAttentionRouter with the Qwen3.6 / Gemma4 / DeepSeek layouts).

The GPU runner reads the layout through ``ModelConfig.attention_layout`` (set by
``layout_for_config``): softmax and global layers attend over the whole context, sliding-window
layers over the last ``window`` tokens (the paged-attention kernels' ``window`` argument), so
a Gemma-style interleaving of local and global layers runs in one decode graph. Gated DeltaNet
and MLA layers are available as reference implementations (``archs.ssm`` / ``archs.mla``); a
runner asked to execute them raises.
"""
from __future__ import annotations

import dataclasses
import enum
from dataclasses import dataclass


class Backend(str, enum.Enum):
    SOFTMAX = "softmax"
    GATED_DELTA_NET = "gated_delta_net"
    SLIDING_WINDOW = "sliding_window"
    GLOBAL_FULL = "global_full"
    MLA = "mla"


@dataclass(frozen=True)
class AttentionBackend:
    kind: Backend
    window: int = 0          # SLIDING_WINDOW only

    @staticmethod
    def softmax() -> "AttentionBackend":
        return AttentionBackend(Backend.SOFTMAX)

    @staticmethod
    def sliding(window: int) -> "AttentionBackend":
        if window <= 0:
            raise ValueError("sliding window must be positive")
        return AttentionBackend(Backend.SLIDING_WINDOW, window)

    @staticmethod
    def global_full() -> "AttentionBackend":
        return AttentionBackend(Backend.GLOBAL_FULL)

    @staticmethod
    def delta_net() -> "AttentionBackend":
        return AttentionBackend(Backend.GATED_DELTA_NET)

    @staticmethod
    def mla() -> "AttentionBackend":
        return AttentionBackend(Backend.MLA)

    @property
    def is_recurrent(self) -> bool:
        return self.kind == Backend.GATED_DELTA_NET

    @property
    def is_mla(self) -> bool:
        return self.kind == Backend.MLA

    @property
    def is_kv_cacheable(self) -> bool:
        return not self.is_recurrent

    @property
    def name(self) -> str:
        return self.kind.value

    def __str__(self) -> str:
        if self.kind == Backend.SLIDING_WINDOW:
            return f"SlidingWindow(w={self.window})"
        return {Backend.SOFTMAX: "Softmax", Backend.GATED_DELTA_NET: "GatedDeltaNet",
                Backend.GLOBAL_FULL: "GlobalFull", Backend.MLA: "MLA"}[self.kind]


class HybridAttentionRouter:
    def __init__(self, layout: list[AttentionBackend]):
        if not layout:
            raise ValueError("HybridAttentionRouter: layout must not be empty")
        self._layout = list(layout)

    @classmethod
    def uniform(cls, n_layers: int, backend: AttentionBackend) -> "HybridAttentionRouter":
        return cls([backend] * n_layers)

    def backend_for_layer(self, layer: int) -> AttentionBackend:
        return self._layout[layer]

    def n_layers(self) -> int:
        return len(self._layout)

    def count(self, backend: AttentionBackend) -> int:
        return sum(1 for b in self._layout if b == backend)

    def layout(self) -> list[AttentionBackend]:
        return list(self._layout)

    def windows(self) -> list[int]:
        """Per-layer attention window for the paged kernels (0 = whole context)."""
        out = []
        for i, b in enumerate(self._layout):
            if b.is_recurrent or b.is_mla:
                raise NotImplementedError(f"layer {i}: {b} runs only in the reference implementations")
            out.append(b.window if b.kind == Backend.SLIDING_WINDOW else 0)
        return out

    # -- layouts of named model families ------------------------------------
    @classmethod
    def qwen3_6(cls, n_layers: int) -> "HybridAttentionRouter":
        """Three gated-DeltaNet layers then one softmax layer, repeated."""
        return cls([AttentionBackend.softmax() if i % 4 == 3 else AttentionBackend.delta_net()
                    for i in range(n_layers)])

    @classmethod
    def qwen3_6_27b(cls) -> "HybridAttentionRouter":
        return cls.qwen3_6(64)

    @classmethod
    def qwen3_6_35b_a3b(cls) -> "HybridAttentionRouter":
        return cls.qwen3_6(96)

    @classmethod
    def gemma4(cls, n_layers: int, sliding_window: int, global_every_n: int) -> "HybridAttentionRouter":
        """Sliding-window layers with a global layer every ``global_every_n`` (the last layer
        is always global)."""
        out = []
        for i in range(n_layers):
            glob = i == n_layers - 1 or (i > 0 and i % global_every_n == global_every_n - 1)
            out.append(AttentionBackend.global_full() if glob else AttentionBackend.sliding(sliding_window))
        return cls(out)

    @classmethod
    def deepseek_v2(cls, n_layers: int) -> "HybridAttentionRouter":
        return cls.uniform(n_layers, AttentionBackend.mla())


def layout_for_config(cfg) -> HybridAttentionRouter:
    """The router a ``ModelConfig`` implies: an explicit ``attention_layout`` (list of
    windows, 0 = global) in ``cfg.extra``; else a uniform sliding window when the GGUF
    metadata names one; else softmax everywhere."""
    lay = cfg.extra.get("attention_layout") if cfg.extra else None
    if lay is not None:
        return HybridAttentionRouter([AttentionBackend.sliding(w) if w else AttentionBackend.global_full()
                                      for w in lay])
    if cfg.sliding_window:
        return HybridAttentionRouter.uniform(cfg.n_layers, AttentionBackend.sliding(cfg.sliding_window))
    return HybridAttentionRouter.uniform(cfg.n_layers, AttentionBackend.softmax())


def with_layout(cfg, router: HybridAttentionRouter):
    """A copy of ``cfg`` whose layers follow ``router`` (windows only)."""
    extra = dict(cfg.extra or {})
    extra["attention_layout"] = router.windows()
    return dataclasses.replace(cfg, extra=extra)
