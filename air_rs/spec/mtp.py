"""Multi-token prediction heads (reference ``src/multi_token.rs``: MtpConfig, MtpHeadWeights,
mtp_head_forward = RMSNorm -> projection (+ optional per-head bias) -> LM head,
mtp_forward_all, mtp_speculative_draft).

``MtpHeads`` exposes the interface ``MedusaDecoder`` drafts from (``n_heads`` and
``logits(h, lm_head_fn)``), so DeepSeek-V3-style MTP heads draft a token chain from the
target's own final hidden state and every draft goes through the target's tree verification:
``MedusaDecoder(engine, MtpHeads(...))``.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class MtpConfig:
    n_extra_heads: int = 1
    vocab_size: int = 102400
    hidden_dim: int = 7168
    enabled_at_inference: bool = True

    @classmethod
    def deepseek_v3(cls) -> "MtpConfig":
        return cls(1, 102400, 7168, True)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    xf = x.float()
    return xf / torch.sqrt((xf * xf).mean(-1, keepdim=True) + eps) * w.float()


@dataclass
class MtpHead:
    norm_weight: torch.Tensor          # [H]
    proj: torch.Tensor                 # [H, H]
    head_bias: torch.Tensor | None = None
    lm_head: torch.Tensor | None = None   # [V, H]; None: the main LM head (tied)

    def forward(self, hidden: torch.Tensor, lm_head_fn=None) -> torch.Tensor:
        x = rms_norm(hidden, self.norm_weight) @ self.proj.float().t()
        if self.head_bias is not None:
            x = x + self.head_bias.float()
        if self.lm_head is not None:
            return x @ self.lm_head.float().t()
        return lm_head_fn(x)


class MtpHeads:
    def __init__(self, heads: list[MtpHead], cfg: MtpConfig | None = None):
        self.heads = heads
        self.cfg = cfg or MtpConfig(n_extra_heads=len(heads))
        self.n_heads = len(heads) if self.cfg.enabled_at_inference else 0

    @classmethod
    def random(cls, hidden: int, n_heads: int = 1, device="cpu", seed: int = 0, scale: float = 0.02):
        g = torch.Generator().manual_seed(seed)
        hs = [MtpHead(torch.ones(hidden, device=device),
                      (torch.eye(hidden) + torch.randn(hidden, hidden, generator=g) * scale).to(device))
              for _ in range(n_heads)]
        return cls(hs, MtpConfig(n_heads, 0, hidden, True))

    def logits(self, h: torch.Tensor, lm_head_fn) -> list[torch.Tensor]:
        """h [S, H] -> logits of tokens t+2, t+3, ... (one [S, V] per head)."""
        if not self.cfg.enabled_at_inference:
            return []
        return [hd.forward(h, lm_head_fn) for hd in self.heads]


def mtp_forward_all(hidden: torch.Tensor, lm_head_fn, heads: MtpHeads):
    """(main logits, [extra logits per head]) of hidden states [..., H]."""
    return lm_head_fn(hidden.float()), heads.logits(hidden, lm_head_fn)


def mtp_speculative_draft(main_logits: torch.Tensor, extra_logits: list[torch.Tensor], sample_fn=None):
    """Main token from the last position's main logits and the draft of the token after it
    from the first MTP head (greedy unless ``sample_fn(logits) -> int`` is given)."""
    pick = sample_fn or (lambda lg: int(torch.argmax(lg)))
    main = pick(main_logits[..., -1, :].reshape(-1))
    draft = pick(extra_logits[0][..., -1, :].reshape(-1)) if extra_logits else None
    return main, draft
