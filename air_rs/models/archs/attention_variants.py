"""Attention variants as reference implementations (reference ``src/ops.rs:1700-2060``):
FP4 (E2M1) micro-scaled Q / K attention, KIMI-style linear attention with the ELU + 1
feature map and causal running state, and per-head sigmoid-gated attention output.

Batched tensor code over [B, S, H, D] (any device); used to evaluate these variants against
the softmax path with the same weights.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

FP4_VALUES = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])
FP4_MAX = 6.0
FP4_BLOCK = 16


def fp4_quantize_blocked(x: torch.Tensor, block: int = FP4_BLOCK) -> tuple[torch.Tensor, torch.Tensor]:
    """Round each value to the nearest E2M1 magnitude after dividing by its block's scale
    (max |x| / 6 over ``block`` consecutive values of the flattened tensor); returns the
    dequantised tensor and the scales. Ties go to the smaller magnitude."""
    flat = x.float().reshape(-1)
    n = flat.numel()
    pad = (-n) % block
    xb = F.pad(flat, (0, pad)).reshape(-1, block)
    amax = xb.abs().amax(-1, keepdim=True)
    scale = torch.where(amax > 0, amax / FP4_MAX, torch.ones_like(amax))
    mag = (xb.abs() / scale)
    vals = FP4_VALUES.to(x.device)
    idx = (mag[..., None] - vals).abs().argmin(-1)
    q = torch.sign(xb) * vals[idx] * scale
    return q.reshape(-1)[:n].reshape(x.shape).to(x.dtype), scale.reshape(-1)


def gqa_attention(q, k, v, causal: bool = True) -> torch.Tensor:
    """q [B, Sq, H, D], k / v [B, Skv, Hkv, D] -> [B, Sq, H, D] softmax attention."""
    rep = q.shape[2] // k.shape[2]
    qh = q.transpose(1, 2).float()
    kh = k.repeat_interleave(rep, 2).transpose(1, 2).float()
    vh = v.repeat_interleave(rep, 2).transpose(1, 2).float()
    mask = None
    if causal and q.shape[1] > 1:
        Sq, Skv = q.shape[1], k.shape[1]
        mask = torch.arange(Skv, device=q.device)[None] <= torch.arange(Sq, device=q.device)[:, None] + (Skv - Sq)
    return F.scaled_dot_product_attention(qh, kh, vh, attn_mask=mask).transpose(1, 2)


def fp4_attention(q, k, v, causal: bool = True) -> torch.Tensor:
    """Softmax attention with Q and K passed through FP4 micro-scaling (SageAttention3-style
    emulation); V stays in full precision."""
    return gqa_attention(fp4_quantize_blocked(q)[0], fp4_quantize_blocked(k)[0], v, causal)


def phi_elu(x: torch.Tensor) -> torch.Tensor:
    return F.elu(x) + 1.0


def linear_attention(q, k, v) -> torch.Tensor:
    """Causal linear attention o_t = phi(q_t) S_t / (phi(q_t) . z_t) with S_t = sum_{j<=t}
    phi(k_j) v_j^T and z_t = sum_{j<=t} phi(k_j); keys and queries aligned at the end when
    Sq < Skv (the first Skv - Sq keys are context for every query). GQA heads shared."""
    rep = q.shape[2] // k.shape[2]
    Sq, Skv = q.shape[1], k.shape[1]
    pq = phi_elu(q.float())
    pk = phi_elu(k.float()).repeat_interleave(rep, 2)
    vv = v.float().repeat_interleave(rep, 2)
    S = torch.cumsum(torch.einsum("bshd,bshe->bshde", pk, vv), 1)[:, Skv - Sq:]
    z = torch.cumsum(pk, 1)[:, Skv - Sq:]
    num = torch.einsum("bshd,bshde->bshe", pq, S)
    den = torch.einsum("bshd,bshd->bsh", pq, z).clamp_min(1e-6)
    return num / den[..., None]


def gated_attention_output(attn_out: torch.Tensor, x: torch.Tensor, w_gate: torch.Tensor | None = None):
    """attn_out [B, S, H, D] scaled per head by sigmoid(gate): the mean of the head's slice
    of x [B, S, H*D] (the reference's parameter-free gate), or ``x @ w_gate^T`` [H, H*D] when
    a learned gate is given."""
    B, S, H, D = attn_out.shape
    if w_gate is None:
        g = x.float().reshape(B, S, H, D).mean(-1)
    else:
        g = x.float() @ w_gate.float().t()
    return attn_out * torch.sigmoid(g)[..., None].to(attn_out.dtype)


def gated_attention(q, k, v, x, w_gate=None, causal: bool = True) -> torch.Tensor:
    return gated_attention_output(gqa_attention(q, k, v, causal), x, w_gate)
