"""Gemma-family pieces (reference ``src/gemma4.rs``, ``src/ops.rs:82-149, 365-448, 2287-2342``):
RMSNorm with (1 + w), tanh-approximate GELU / GeGLU, logit soft-capping in attention, and the
sigmoid top-k MoE router with weighted sum."""
from __future__ import annotations

import math

import torch


def gemma_rms_norm(x, w, eps=1e-6):
    xf = x.float()
    return xf / torch.sqrt((xf * xf).mean(-1, keepdim=True) + eps) * (1.0 + w.float())


def gelu_tanh(x):
    return 0.5 * x * (1.0 + torch.tanh(math.sqrt(2.0 / math.pi) * (x + 0.044715 * x ** 3)))


def geglu_ffn(x, w_gate, w_up, w_down):
    return (gelu_tanh(x @ w_gate.t()) * (x @ w_up.t())) @ w_down.t()


def softcap(s, cap: float):
    return cap * torch.tanh(s / cap)


def softcapped_attention(q, k, v, cap: float = 50.0, causal: bool = True):
    """q [Lq, h, d], k/v [Lk, h, d]."""
    s = softcap(torch.einsum("qhd,khd->hqk", q, k) / math.sqrt(q.shape[-1]), cap)
    if causal:
        Lq, Lk = q.shape[0], k.shape[0]
        s = s.masked_fill(torch.triu(torch.ones(Lq, Lk, dtype=torch.bool), 1 + Lk - Lq)[None], float("-inf"))
    return torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), v)


def sigmoid_moe_route(logits, k: int, normalize: bool = True):
    """Sigmoid scores, top-k experts, optionally renormalised: (ids [T, k], weights [T, k])."""
    s = torch.sigmoid(logits.float())
    w, ids = torch.topk(s, k, -1)
    if normalize:
        w = w / w.sum(-1, keepdim=True).clamp_min(1e-9)
    return ids, w


def moe_weighted_sum(expert_out, ids, w):
    """expert_out [T, E, H] -> sum_j w[t, j] * expert_out[t, ids[t, j]]."""
    g = torch.gather(expert_out, 1, ids[..., None].expand(-1, -1, expert_out.shape[-1]))
    return (g * w[..., None]).sum(1)
