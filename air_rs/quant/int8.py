"""W8A8 int8 GEMM and symmetric int8 quantisation (reference ``src/w8a8.rs``), and the Q8_0 KV
block codec (reference ``src/kv_cache.rs:26-109``: 32-element blocks, scale = absmax/127).

``w8a8_matmul`` takes per-tensor scales s = absmax/127 (what ``quantize_f32_to_i8`` returns)
and computes acc_int32 * s_x * s_w; the reference divides once more by 127^2, which is only
consistent if its callers pass absmax itself, so the scale convention is stated here.
"""
from __future__ import annotations

import torch


def quantize_f32_to_i8(x: torch.Tensor) -> tuple[torch.Tensor, float]:
    amax = float(x.abs().max()) if x.numel() else 0.0
    if amax == 0.0:
        return torch.zeros_like(x, dtype=torch.int8), 1.0
    s = amax / 127.0
    return torch.clamp(torch.round(x / s), -127, 127).to(torch.int8), s


def w8a8_matmul(xq: torch.Tensor, wq: torch.Tensor, sx: float, sw: float) -> torch.Tensor:
    """[M, K] int8 x [K, N] int8 -> f32 [M, N] with int32 accumulation."""
    acc = xq.to(torch.int32) @ wq.to(torch.int32)
    return acc.float() * (sx * sw)


def kv_q8_0_encode(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """x [..., D] (D % 32 == 0) -> (int8 codes, f32 scales [..., D/32])."""
    b = x.float().reshape(*x.shape[:-1], -1, 32)
    s = b.abs().amax(-1) / 127.0
    q = torch.where(s[..., None] > 0, torch.round(b / s[..., None].clamp_min(1e-30)), torch.zeros_like(b))
    return q.clamp(-127, 127).to(torch.int8).reshape(x.shape), s


def kv_q8_0_decode(q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    return (q.float().reshape(*q.shape[:-1], -1, 32) * s[..., None]).reshape(q.shape)
