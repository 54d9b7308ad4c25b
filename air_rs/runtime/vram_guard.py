"""VRAM guard (reference ``src/vram_guard.rs``): refuse a load whose estimated device
footprint (weights + KV pool + activation workspace) exceeds a fraction (default 80 %) of
the GPU's memory.
"""
from __future__ import annotations

import os
from dataclasses import dataclass

VRAM_CAP_FRACTION = float(os.environ.get("AIR_VRAM_FRACTION", os.environ.get("AIR_VRAM_CAP_FRACTION", "0.80")))


def set_default_fraction(frac: float):
    """Cap used by later loads (the KV planner and ``VramBudget.check`` defaults)."""
    global VRAM_CAP_FRACTION
    if not 0.0 < frac <= 1.0:
        raise ValueError("VRAM cap fraction must be in (0, 1]")
    VRAM_CAP_FRACTION = float(frac)


def default_fraction() -> float:
    return VRAM_CAP_FRACTION


@dataclass
class VramCheckResult:
    kind: str                  # "accept" | "reject" | "skipped"
    estimate_bytes: int = 0
    cap_bytes: int = 0

    @property
    def shortfall_bytes(self) -> int:
        return max(0, self.estimate_bytes - self.cap_bytes)

    def ok_to_load(self) -> bool:
        return self.kind != "reject"

    def summary(self) -> str:
        if self.kind == "accept":
            return "VRAM guard: load accepted"
        if self.kind == "skipped":
            return "VRAM guard: skipped (no CUDA device or query failed)"
        mib = 1 << 20
        return (f"VRAM guard: load rejected - need {self.estimate_bytes / mib:.0f} MiB, cap "
                f"{self.cap_bytes / mib:.0f} MiB (shortfall {self.shortfall_bytes / mib:.0f} MiB). "
                f"Reduce the context length / KV pool or use a smaller quant.")


@dataclass
class VramBudget:
    total_bytes: int
    free_bytes: int
    estimate_bytes: int
    cap_fraction: float | None = None

    def __post_init__(self):
        if self.cap_fraction is None:
            self.cap_fraction = VRAM_CAP_FRACTION

    @property
    def cap_bytes(self) -> int:
        return int(self.total_bytes * self.cap_fraction)

    @staticmethod
    def estimate(weight_bytes: int, n_layers: int, n_kv_heads: int, head_dim: int, kv_tokens: int,
                 kv_dtype_bytes: int = 2, workspace_bytes: int = 512 << 20) -> int:
        kv = 2 * n_layers * n_kv_heads * head_dim * kv_tokens * kv_dtype_bytes
        return weight_bytes + kv + workspace_bytes

    @staticmethod
    def query(device=0, mem_get_info=None) -> tuple[int, int] | None:
        """(free, total) bytes of the device; ``mem_get_info`` can be injected (tests)."""
        try:
            if mem_get_info is not None:
                return mem_get_info(device)
            import torch
            if not torch.cuda.is_available():
                return None
            return torch.cuda.mem_get_info(device)
        except Exception:
            return None

    @classmethod
    def check(cls, estimate_bytes: int, device=0, cap_fraction: float | None = None,
              mem_get_info=None) -> VramCheckResult:
        q = cls.query(device, mem_get_info)
        if q is None:
            return VramCheckResult("skipped", estimate_bytes)
        free, total = q
        b = cls(total, free, estimate_bytes, cap_fraction)
        kind = "accept" if estimate_bytes <= b.cap_bytes else "reject"
        return VramCheckResult(kind, estimate_bytes, b.cap_bytes)
