"""FP8 (E4M3) rows of the paged KV pool, on the host side.

A pool built with ``kv_dtype="fp8"`` is a uint8 tensor ``[L, num_blocks, 2, n_kv, block,
head_dim + 16]``; each (token, KV head) row holds ``head_dim`` E4M3 codes, the row's scale
``s = max|x| / 448`` as f32, and 12 zero bytes that keep rows 16-byte aligned for the
kernels' 16-byte copies. ``x ~= s * code``. The RoPE/KV-write kernel produces these rows on
the GPU; this module is the torch statement of the same format, used to fill or read a pool
from the host (tests, snapshots of a bf16 run replayed into an fp8 pool) and as the oracle.

Reference: Q8_0 quantisation of the host KV cache (``src/kv_cache.rs:54-92``: int8 codes,
one f16 scale per 32 values). Here one scale per head row and E4M3 codes, which the tensor
path converts exactly to f16.
"""
from __future__ import annotations

import torch

E4M3_MAX = 448.0
PAD = 16


def row_bytes(head_dim: int) -> int:
    return head_dim + PAD


def quantize_rows(x: torch.Tensor) -> torch.Tensor:
    """[..., D] float -> [..., D + 16] uint8 (codes, f32 scale, zero padding)."""
    xf = x.float()
    d = xf.shape[-1]
    amax = xf.abs().amax(-1, keepdim=True)
    s = amax / E4M3_MAX
    inv = torch.where(s > 0, 1.0 / s, torch.zeros_like(s))
    codes = (xf * inv).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn).view(torch.uint8)
    out = torch.zeros(*xf.shape[:-1], d + PAD, dtype=torch.uint8, device=x.device)
    out[..., :d] = codes
    out[..., d:d + 4] = s.contiguous().view(torch.uint8)
    return out


def dequantize_rows(q: torch.Tensor) -> torch.Tensor:
    """[..., D + 16] uint8 -> [..., D] float32."""
    d = q.shape[-1] - PAD
    codes = q[..., :d].contiguous().view(torch.float8_e4m3fn).float()
    s = q[..., d:d + 4].contiguous().view(torch.float32)
    return codes * s


def pool_dequantize(kv: torch.Tensor) -> torch.Tensor:
    """A whole fp8 pool (any leading dims) -> float32 values with the bf16 pool's shape."""
    return dequantize_rows(kv)
