"""RoPE variants (reference ``src/ops.rs:643-690, 945-1133, 1276-1420``, ``src/yarn.rs``,
``src/dual_rope.rs``): partial rotary, GPT-J interleaved pairs, Llama-3.1 frequency scaling,
YaRN (NTK-by-parts interpolation + attention temperature), dual local/global theta, ALiBi
slopes and sinusoidal absolute positions."""
from __future__ import annotations

import math

import torch


def inv_freq(dim: int, theta: float) -> torch.Tensor:
    return 1.0 / torch.pow(torch.tensor(float(theta)), torch.arange(0, dim, 2, dtype=torch.float32) / dim)


def rope_neox(x: torch.Tensor, pos: torch.Tensor, freqs: torch.Tensor, rot_dim: int | None = None) -> torch.Tensor:
    """Half-split rotation of the first ``rot_dim`` features (partial rotary keeps the rest)."""
    d = x.shape[-1]
    r = rot_dim or d
    ang = pos.float()[:, None] * freqs[None, : r // 2]
    c, s = torch.cos(ang), torch.sin(ang)
    while c.dim() < x.dim():
        c, s = c.unsqueeze(-2), s.unsqueeze(-2)
    x1, x2, rest = x[..., : r // 2], x[..., r // 2: r], x[..., r:]
    return torch.cat([x1 * c - x2 * s, x1 * s + x2 * c, rest], -1)


def rope_interleaved(x: torch.Tensor, pos: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    """GPT-J style: pairs (2i, 2i+1) rotate together."""
    ang = pos.float()[:, None] * freqs[None, :]
    c, s = torch.cos(ang), torch.sin(ang)
    while c.dim() < x.dim():
        c, s = c.unsqueeze(-2), s.unsqueeze(-2)
    xe, xo = x[..., 0::2], x[..., 1::2]
    out = torch.stack([xe * c - xo * s, xe * s + xo * c], -1)
    return out.flatten(-2)


def llama3_scaled_freqs(freqs: torch.Tensor, factor: float = 8.0, low_freq_factor: float = 1.0,
                        high_freq_factor: float = 4.0, original_max_pos: int = 8192) -> torch.Tensor:
    """Llama-3.1 rope scaling: long wavelengths divided by ``factor``, short ones kept, a smooth
    blend in between."""
    low_wl = original_max_pos / low_freq_factor
    high_wl = original_max_pos / high_freq_factor
    wl = 2 * math.pi / freqs
    smooth = (original_max_pos / wl - low_freq_factor) / (high_freq_factor - low_freq_factor)
    scaled = torch.where(wl > low_wl, freqs / factor, freqs)
    mid = (wl <= low_wl) & (wl >= high_wl)
    return torch.where(mid, (1 - smooth) * freqs / factor + smooth * freqs, scaled)


class YarnFrequencies:
    """YaRN: per-dimension blend of interpolated (freq / s) and extrapolated frequencies by
    the number of rotations a dimension makes over the original context, plus the
    attention-logit temperature 0.1 ln(s) + 1."""

    def __init__(self, dim: int, theta: float, scale: float, original_max_pos: int, beta_fast: float = 32.0,
                 beta_slow: float = 1.0):
        self.dim, self.theta, self.scale = dim, theta, scale
        f = inv_freq(dim, theta)
        if scale <= 1.0:
            self.freqs, self.mscale = f, 1.0
            return

        def corr_dim(n_rot):
            return dim * math.log(original_max_pos / (n_rot * 2 * math.pi)) / (2 * math.log(theta))
        lo = max(math.floor(corr_dim(beta_fast)), 0)
        hi = min(math.ceil(corr_dim(beta_slow)), dim // 2 - 1)
        ramp = ((torch.arange(dim // 2, dtype=torch.float32) - lo) / max(hi - lo, 1e-3)).clamp(0, 1)
        extrap_w = 1.0 - ramp                       # 1 = keep (high frequency), 0 = interpolate
        self.freqs = f / scale * (1 - extrap_w) + f * extrap_w
        self.mscale = 0.1 * math.log(scale) + 1.0


def dual_rope_freqs(dim: int, local_theta: float, global_theta: float) -> tuple[torch.Tensor, torch.Tensor]:
    """Separate caches for sliding-window (local) and global layers (Gemma-style)."""
    return inv_freq(dim, local_theta), inv_freq(dim, global_theta)


def alibi_slopes(n_heads: int) -> torch.Tensor:
    def pow2(n):
        start = 2 ** (-(2 ** -(math.log2(n) - 3)))
        return [start * start ** i for i in range(n)]
    if math.log2(n_heads).is_integer():
        return torch.tensor(pow2(n_heads))
    m = 2 ** math.floor(math.log2(n_heads))
    return torch.tensor(pow2(m) + pow2(2 * m)[0::2][: n_heads - m])


def sinusoidal_positions(n_pos: int, dim: int) -> torch.Tensor:
    pos = torch.arange(n_pos, dtype=torch.float32)[:, None]
    div = torch.exp(torch.arange(0, dim, 2, dtype=torch.float32) * (-math.log(10000.0) / dim))
    pe = torch.zeros(n_pos, dim)
    pe[:, 0::2] = torch.sin(pos * div)
    pe[:, 1::2] = torch.cos(pos * div)
    return pe
