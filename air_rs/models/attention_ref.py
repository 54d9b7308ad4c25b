"""Reference attention algorithms that the GPU kernels restate (reference
``src/flash_decode.rs``: split-K flash decoding with per-chunk (m, l, o) and a log-sum-exp
merge; ``src/chunked_attn.rs``: blockwise online-softmax attention with GQA and causal masking,
peak-memory estimate).

These are the oracles for the paged kernels: the decode kernel is split-K over CTAs with the
same per-split statistics and merge (``csrc/attention*.cu``), and the prefill kernel is the
blockwise online softmax over KV tiles. Written as batched tensor code (any device).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

DEFAULT_CHUNK_SIZE = 64
DEFAULT_BLOCK_SIZE = 512


@dataclass
class ChunkOutput:
    m: torch.Tensor      # [H] running max of the scaled scores
    l: torch.Tensor      # [H] sum of exp(score - m)
    o: torch.Tensor      # [H, D] sum of exp(score - m) * v (unnormalised)


def chunk_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float) -> ChunkOutput:
    """One split: q [H, D] against this chunk's k / v [T, H, D] (already head-expanded)."""
    s = torch.einsum("hd,thd->ht", q.float(), k.float()) * scale
    m = s.amax(-1)
    p = torch.exp(s - m[:, None])
    return ChunkOutput(m, p.sum(-1), torch.einsum("ht,thd->hd", p, v.float()))


def reduce_chunks(chunks: list[ChunkOutput]) -> torch.Tensor:
    """Log-sum-exp merge of split partials -> [H, D]."""
    M = torch.stack([c.m for c in chunks]).amax(0)
    L = torch.zeros_like(M)
    O = torch.zeros_like(chunks[0].o)
    for c in chunks:
        f = torch.exp(c.m - M)
        L = L + c.l * f
        O = O + c.o * f[:, None]
    return O / L[:, None]


def flash_decode(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, chunk: int = DEFAULT_CHUNK_SIZE) -> torch.Tensor:
    """Decode attention of one query row q [H, D] over k / v [T, Hkv, D] (GQA), split into
    ``chunk``-token pieces."""
    H, D = q.shape
    rep = H // k.shape[1]
    kk, vv = k.repeat_interleave(rep, 1), v.repeat_interleave(rep, 1)
    scale = 1.0 / math.sqrt(D)
    parts = [chunk_attention(q, kk[t:t + chunk], vv[t:t + chunk], scale) for t in range(0, k.shape[0], chunk)]
    return reduce_chunks(parts)


def reference_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """Dense softmax attention of one query row (the oracle for ``flash_decode``)."""
    H, D = q.shape
    rep = H // k.shape[1]
    kk, vv = k.repeat_interleave(rep, 1).float(), v.repeat_interleave(rep, 1).float()
    p = torch.softmax(torch.einsum("hd,thd->ht", q.float(), kk) / math.sqrt(D), -1)
    return torch.einsum("ht,thd->hd", p, vv)


def max_abs_error(a: torch.Tensor, b: torch.Tensor) -> float:
    return float((a.float() - b.float()).abs().max())


@dataclass
class ChunkedAttentionConfig:
    block_size: int = DEFAULT_BLOCK_SIZE
    n_heads: int = 32
    n_kv_heads: int = 8
    head_dim: int = 128
    causal: bool = True

    def gqa_groups(self) -> int:
        if self.n_heads % self.n_kv_heads:
            raise ValueError("n_heads must be divisible by n_kv_heads")
        return self.n_heads // self.n_kv_heads

    def scale(self) -> float:
        return 1.0 / math.sqrt(self.head_dim)

    def validate(self):
        if self.block_size <= 0:
            raise ValueError("block_size must be > 0")
        if self.head_dim <= 0:
            raise ValueError("head_dim must be > 0")
        if self.n_heads < self.n_kv_heads or self.n_heads % self.n_kv_heads:
            raise ValueError("n_heads must be a multiple of n_kv_heads")


def blockwise_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cfg: ChunkedAttentionConfig) -> torch.Tensor:
    """q [Sq, H, D], k / v [Skv, Hkv, D] -> [Sq, H, D] with an online softmax over KV blocks
    of ``cfg.block_size`` (memory O(Sq * block) instead of O(Sq * Skv)); causal rule: key j is
    visible to query i iff j <= i + (Skv - Sq)."""
    cfg.validate()
    Sq, H, D = q.shape
    Skv = k.shape[0]
    rep = cfg.gqa_groups()
    qf = q.float() * cfg.scale()
    m = torch.full((H, Sq), float("-inf"))
    l = torch.zeros(H, Sq)
    o = torch.zeros(H, Sq, D)
    qi = torch.arange(Sq)[:, None] + (Skv - Sq)
    for b0 in range(0, Skv, cfg.block_size):
        kb = k[b0:b0 + cfg.block_size].float().repeat_interleave(rep, 1)
        vb = v[b0:b0 + cfg.block_size].float().repeat_interleave(rep, 1)
        s = torch.einsum("shd,thd->hst", qf, kb)
        if cfg.causal:
            kj = torch.arange(b0, b0 + kb.shape[0])[None, :]
            s = s.masked_fill(~(kj <= qi)[None], float("-inf"))
        m_new = torch.maximum(m, s.amax(-1))
        safe = torch.where(torch.isinf(m_new), torch.zeros_like(m_new), m_new)
        corr = torch.exp(m - safe)
        p = torch.exp(s - safe[..., None])
        l = l * corr + p.sum(-1)
        o = o * corr[..., None] + torch.einsum("hst,thd->hsd", p, vb)
        m = m_new
    out = o / l.clamp_min(1e-30)[..., None]
    return out.transpose(0, 1)


def peak_memory_bytes(seq_q: int, seq_kv: int, cfg: ChunkedAttentionConfig) -> int:
    """Score-matrix bytes of the blockwise method: seq_q x min(block, seq_kv) x heads x 4."""
    return seq_q * min(cfg.block_size, seq_kv) * cfg.n_heads * 4


def memory_reduction_factor(seq_q: int, seq_kv: int, cfg: ChunkedAttentionConfig) -> float:
    block = seq_q * min(cfg.block_size, seq_kv) * cfg.n_heads
    full = seq_q * seq_kv * cfg.n_heads
    return 1.0 if full == 0 else full / block
