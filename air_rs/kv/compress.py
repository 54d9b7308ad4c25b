"""KV compression codecs for a warm tier (reference ``src/kv_compress.rs``: 1-bit mean-centred
sign keys, 8-bit affine values, QJL 1-bit random-projection keys with a Hamming-distance
similarity estimate, attention / recency / prefix triage scores, KV budget arithmetic).

All codecs are batched tensor code over rows of [N, head_dim] (any device): a warm tier
compresses whole evicted blocks at once, and QJL scores every cached key against a query
with one XOR-popcount pass to pick the blocks worth restoring.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

BF16_BYTES = 2
KEY_COMPRESSION_RATIO = 16.0
VALUE_COMPRESSION_RATIO = 2.0
QJL_PROJ_DIM = 64

_POP8 = torch.tensor([bin(i).count("1") for i in range(256)], dtype=torch.int32)


def _packbits(bits: torch.Tensor) -> torch.Tensor:
    """bool [..., n] -> uint8 [..., ceil(n/8)], bit i of byte j = element 8j + i."""
    n = bits.shape[-1]
    pad = (-n) % 8
    if pad:
        bits = torch.nn.functional.pad(bits, (0, pad))
    w = (1 << torch.arange(8, device=bits.device)).to(torch.int32)
    return (bits.reshape(*bits.shape[:-1], -1, 8).to(torch.int32) * w).sum(-1).to(torch.uint8)


def _unpackbits(packed: torch.Tensor, n: int) -> torch.Tensor:
    b = (packed[..., None].to(torch.int32) >> torch.arange(8, device=packed.device)) & 1
    return b.reshape(*packed.shape[:-1], -1)[..., :n].bool()


# ---------------------------------------------------------------------------- 1-bit keys
@dataclass
class CompressedKeys:
    sign_bits: torch.Tensor      # uint8 [N, d/8]: 1 where k_i >= mean
    magnitude: torch.Tensor      # [N] L2 norm
    mean: torch.Tensor           # [N]
    dim: int

    @classmethod
    def compress(cls, k: torch.Tensor) -> "CompressedKeys":
        kf = k.float()
        mean = kf.mean(-1)
        return cls(_packbits(kf >= mean[:, None]), kf.norm(dim=-1), mean, k.shape[-1])

    def decompress(self) -> torch.Tensor:
        sign = _unpackbits(self.sign_bits, self.dim).float() * 2 - 1
        return sign * (self.magnitude / math.sqrt(self.dim))[:, None] + self.mean[:, None]

    def size_bytes(self) -> int:
        return self.sign_bits.numel() + 8 * self.magnitude.numel()

    def uncompressed_bytes(self) -> int:
        return self.magnitude.numel() * self.dim * BF16_BYTES

    def compression_ratio(self) -> float:
        return self.uncompressed_bytes() / max(1, self.size_bytes())


# ---------------------------------------------------------------------------- 8-bit values
@dataclass
class CompressedValues:
    data: torch.Tensor           # uint8 [N, d]
    scale: torch.Tensor          # [N] (max - min) / 255 (1 when constant)
    min_val: torch.Tensor        # [N]

    @classmethod
    def compress(cls, v: torch.Tensor) -> "CompressedValues":
        vf = v.float()
        lo, hi = vf.amin(-1), vf.amax(-1)
        rng = hi - lo
        scale = torch.where(rng > 0, rng / 255.0, torch.ones_like(rng))
        q = torch.round((vf - lo[:, None]) / scale[:, None]).clamp(0, 255).to(torch.uint8)
        return cls(q, scale, lo)

    def decompress(self) -> torch.Tensor:
        return self.data.float() * self.scale[:, None] + self.min_val[:, None]

    def size_bytes(self) -> int:
        return self.data.numel() + 8 * self.scale.numel()

    def uncompressed_bytes(self) -> int:
        return self.data.numel() * BF16_BYTES

    def compression_ratio(self) -> float:
        return self.uncompressed_bytes() / max(1, self.size_bytes())


# ---------------------------------------------------------------------------- QJL keys
def qjl_projection_matrix(proj_dim: int, orig_dim: int, seed: int = 0, device=None) -> torch.Tensor:
    """Seeded N(0, 1/proj_dim) Gaussian projection [proj_dim, orig_dim]."""
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(proj_dim, orig_dim, generator=g) / math.sqrt(proj_dim)).to(device)


@dataclass
class QjlKeys:
    bits: torch.Tensor           # uint8 [N, m/8]: sign of each projection
    magnitude: torch.Tensor      # [N]
    proj_dim: int

    @classmethod
    def compress(cls, k: torch.Tensor, proj: torch.Tensor) -> "QjlKeys":
        kf = k.float()
        return cls(_packbits((kf @ proj.t()) > 0), kf.norm(dim=-1), proj.shape[0])

    @staticmethod
    def query_bits(q: torch.Tensor, proj: torch.Tensor) -> torch.Tensor:
        return _packbits((q.float() @ proj.t()) > 0)

    def hamming(self, qbits: torch.Tensor) -> torch.Tensor:
        x = torch.bitwise_xor(self.bits, qbits.reshape(1, -1))
        return _POP8.to(x.device)[x.long()].sum(-1)

    def approx_cos_sim(self, qbits: torch.Tensor) -> torch.Tensor:
        """cos(pi * hamming / m): the sign-random-projection estimate of the angle."""
        return torch.cos(math.pi * self.hamming(qbits).float() / self.proj_dim)

    def approx_dot(self, qbits: torch.Tensor, q_norm: float) -> torch.Tensor:
        return self.approx_cos_sim(qbits) * self.magnitude * q_norm

    def size_bytes(self) -> int:
        return self.bits.numel() + 4 * self.magnitude.numel()


# ---------------------------------------------------------------------------- triage
@dataclass
class TriageWeights:
    alpha: float = 0.50          # mean attention received
    beta: float = 0.30           # recency, e^(-lambda * steps since last access)
    gamma: float = 0.20          # prefix bonus
    lam: float = 0.1
    attention_window: int = 16
    prefix_tokens: int = 64


def triage_score(w: TriageWeights, mean_attention, current_step: int, last_access_step, position):
    a = torch.as_tensor(mean_attention, dtype=torch.float64)
    steps = (current_step - torch.as_tensor(last_access_step, dtype=torch.float64)).clamp_min(0)
    r = torch.exp(-w.lam * steps)
    p = (torch.as_tensor(position) < w.prefix_tokens).to(torch.float64)
    return w.alpha * a + w.beta * r + w.gamma * p


def rank_entries(w: TriageWeights, entries: list[tuple[int, float, int]], current_step: int):
    """[(position, mean attention, last access step)] -> [(position, score)] best first."""
    if not entries:
        return []
    pos, att, last = zip(*entries)
    s = triage_score(w, list(att), current_step, list(last), list(pos))
    order = torch.argsort(s, descending=True, stable=True)
    return [(pos[i], float(s[i])) for i in order.tolist()]


# ---------------------------------------------------------------------------- budgets
@dataclass
class KvBudgetCalc:
    n_layers: int = 80
    n_kv_heads: int = 8
    head_dim: int = 128

    def bytes_per_token_per_layer(self, dtype_bytes: int = BF16_BYTES) -> int:
        return 2 * self.n_kv_heads * self.head_dim * dtype_bytes

    def bytes_per_token(self, dtype_bytes: int = BF16_BYTES) -> int:
        return self.n_layers * self.bytes_per_token_per_layer(dtype_bytes)

    def total_bytes(self, context_len: int, dtype_bytes: int = BF16_BYTES) -> int:
        return context_len * self.bytes_per_token(dtype_bytes)

    def total_mb(self, context_len: int, dtype_bytes: int = BF16_BYTES) -> float:
        return self.total_bytes(context_len, dtype_bytes) / 2**20

    def compressed_warm_mb(self, context_len: int) -> float:
        """1-bit keys + 8-bit values (plus per-row scalars)."""
        per = self.n_layers * self.n_kv_heads * (self.head_dim / 8 + 8 + self.head_dim + 8)
        return context_len * per / 2**20

    def fits(self, context_len: int, budget_mb: float, compressed: bool = False) -> bool:
        need = self.compressed_warm_mb(context_len) if compressed else self.total_mb(context_len)
        return need <= budget_mb
