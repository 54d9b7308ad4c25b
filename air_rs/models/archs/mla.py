"""Multi-head latent attention (DeepSeek-V2/V3; reference ``src/mla.rs``): the KV cache holds
one compressed latent c_kv (d_c) plus one shared RoPE key (d_r) per token instead of per-head
K and V. ``mla_forward`` computes attention the explicit way (up-project K/V per head) and
``mla_forward_absorbed`` the decode way (W_uk folded into the query, W_uv applied after the
weighted sum over latents); both must agree."""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from .rope_ext import inv_freq, rope_neox


@dataclass
class MlaWeights:
    w_dq: torch.Tensor      # [d_cq, H]
    w_uq: torch.Tensor      # [nh, d_nope, d_cq]
    w_qr: torch.Tensor      # [nh, d_r, d_cq]
    w_dkv: torch.Tensor     # [d_c, H]
    w_kr: torch.Tensor      # [d_r, H]
    w_uk: torch.Tensor      # [nh, d_nope, d_c]
    w_uv: torch.Tensor      # [nh, d_v, d_c]
    w_o: torch.Tensor       # [H, nh * d_v]

    @classmethod
    def random(cls, H=64, nh=4, d_c=16, d_cq=24, d_nope=8, d_r=4, d_v=8, seed=0):
        g = torch.Generator().manual_seed(seed)
        r = lambda *s: torch.randn(*s, generator=g) * 0.2
        return cls(r(d_cq, H), r(nh, d_nope, d_cq), r(nh, d_r, d_cq), r(d_c, H), r(d_r, H), r(nh, d_nope, d_c),
                   r(nh, d_v, d_c), r(H, nh * d_v))


def latent_cache(w: MlaWeights, x: torch.Tensor, pos: torch.Tensor, theta=10000.0):
    """Per-token cache entries: c_kv [L, d_c] and the RoPE'd shared key [L, d_r]."""
    c = x @ w.w_dkv.t()
    kr = rope_neox((x @ w.w_kr.t())[:, None, :], pos, inv_freq(w.w_kr.shape[0], theta))[:, 0]
    return c, kr


def _queries(w, x, pos, theta):
    cq = x @ w.w_dq.t()
    qn = torch.einsum("hnc,lc->lhn", w.w_uq, cq)
    qr = rope_neox(torch.einsum("hrc,lc->lhr", w.w_qr, cq), pos, inv_freq(w.w_qr.shape[1], theta))
    return qn, qr


def mla_forward(w: MlaWeights, x: torch.Tensor, pos: torch.Tensor, causal=True, theta=10000.0):
    c, kr = latent_cache(w, x, pos, theta)
    qn, qr = _queries(w, x, pos, theta)
    kn = torch.einsum("hnc,lc->lhn", w.w_uk, c)
    v = torch.einsum("hvc,lc->lhv", w.w_uv, c)
    scale = 1.0 / math.sqrt(qn.shape[-1] + qr.shape[-1])
    s = (torch.einsum("qhn,khn->hqk", qn, kn) + torch.einsum("qhr,kr->hqk", qr, kr)) * scale
    if causal:
        L = x.shape[0]
        s = s.masked_fill(torch.triu(torch.ones(L, L, dtype=torch.bool), 1)[None], float("-inf"))
    o = torch.einsum("hqk,khv->qhv", torch.softmax(s, -1), v)
    return o.reshape(x.shape[0], -1) @ w.w_o.t()


def mla_forward_absorbed(w: MlaWeights, x: torch.Tensor, pos: torch.Tensor, cache=None, causal=True,
                         theta=10000.0):
    """Attention over the latent cache: q_lat = W_uk^T q_nope, scores = q_lat . c + q_rope . k_r,
    output = W_uv (sum p c)."""
    c, kr = latent_cache(w, x, pos, theta) if cache is None else cache
    qn, qr = _queries(w, x, pos, theta)
    q_lat = torch.einsum("hnc,qhn->qhc", w.w_uk, qn)
    scale = 1.0 / math.sqrt(qn.shape[-1] + qr.shape[-1])
    s = (torch.einsum("qhc,kc->hqk", q_lat, c) + torch.einsum("qhr,kr->hqk", qr, kr)) * scale
    if causal:
        L = x.shape[0]
        s = s.masked_fill(torch.triu(torch.ones(L, c.shape[0], dtype=torch.bool), 1 + c.shape[0] - L)[None],
                          float("-inf"))
    lat = torch.einsum("hqk,kc->qhc", torch.softmax(s, -1), c)
    o = torch.einsum("hvc,qhc->qhv", w.w_uv, lat)
    return o.reshape(x.shape[0], -1) @ w.w_o.t()
