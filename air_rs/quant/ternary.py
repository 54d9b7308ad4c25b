"""Ternary (BitNet b1.58) weights (reference ``src/ternary.rs``): five trits per byte in base 3
(trit t -> t + 1, first trit least significant), per-row scales, and an int8-activation
matmul that only adds and subtracts.
"""
from __future__ import annotations

import torch

_POW3 = torch.tensor([1, 3, 9, 27, 81], dtype=torch.int32)


def pack_trits(trits: torch.Tensor) -> torch.Tensor:
    """[..., n] in {-1, 0, 1} -> [..., ceil(n/5)] uint8 (padding trits are 0)."""
    t = trits.to(torch.int32) + 1
    n = t.shape[-1]
    pad = (-n) % 5
    if pad:
        t = torch.cat([t, torch.ones(*t.shape[:-1], pad, dtype=torch.int32)], -1)
    t = t.reshape(*t.shape[:-1], -1, 5)
    return (t * _POW3).sum(-1).to(torch.uint8)


def unpack_trits(packed: torch.Tensor, n: int) -> torch.Tensor:
    v = packed.to(torch.int32)[..., None]
    t = (v // _POW3) % 3 - 1
    return t.reshape(*packed.shape[:-1], -1)[..., :n].to(torch.int8)


def quantize_ternary(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """absmean ternarisation per row: scale = mean|w|, trit = round(clamp(w/scale, -1, 1))."""
    s = w.abs().mean(-1).clamp_min(1e-8)
    return torch.clamp(torch.round(w / s[:, None]), -1, 1).to(torch.int8), s


class TernaryMatMul:
    def __init__(self, packed: torch.Tensor, rows: int, cols: int, scales: torch.Tensor):
        self.trits = unpack_trits(packed, cols)[:rows]
        self.rows, self.cols, self.scales = rows, cols, scales.float()

    @classmethod
    def from_float(cls, w: torch.Tensor) -> "TernaryMatMul":
        t, s = quantize_ternary(w)
        return cls(pack_trits(t), w.shape[0], w.shape[1], s)

    def matmul_i8(self, xq: torch.Tensor, sx: float) -> torch.Tensor:
        """x int8 [B, cols] (scale sx) -> f32 [B, rows]: sum of +x and -x by trit sign."""
        pos = (self.trits == 1).to(torch.int32)
        neg = (self.trits == -1).to(torch.int32)
        acc = xq.to(torch.int32) @ (pos - neg).t()
        return acc.float() * sx * self.scales[None, :]
