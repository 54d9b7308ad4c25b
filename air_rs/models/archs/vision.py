"""Vision encoders for multimodal prompts: CLIP / SigLIP ViT (reference ``src/vision.rs``:
VisionConfig presets, PatchEmbedding, pre-norm ViT layers with tanh-GELU MLPs, CLS handling,
vision->language projection, ImageNet / SigLIP normalisation).

Everything runs as batched tensor ops on the encoder's device (on a GPU the matmuls and the
bidirectional attention go to cuBLAS / the fused SDPA kernel). ``image_prompt_hidden`` splices
the projected patch tokens into a prompt's token embeddings at placeholder positions, and
``ModelRunner.prefill(hidden_in=...)`` runs the language model from those embeddings, so a
LLaVA-style image+text prompt goes through the same paged-KV prefill as text.
"""
from __future__ import annotations

import enum
import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F


class VisionEncoderType(str, enum.Enum):
    CLIP_VIT = "clip_vit"
    SIGLIP = "siglip"
    QWEN_VL = "qwen_vl"


@dataclass
class VisionConfig:
    encoder_type: VisionEncoderType
    image_size: int
    patch_size: int
    n_layers: int
    n_heads: int
    hidden_dim: int
    mlp_dim: int
    proj_dim: int
    use_cls_token: bool

    @property
    def num_patches(self) -> int:
        return (self.image_size // self.patch_size) ** 2

    @classmethod
    def clip_vit_l_336(cls) -> "VisionConfig":
        """CLIP ViT-L/14 at 336 px (LLaVA 1.5 / 1.6): 576 patches, CLS token."""
        return cls(VisionEncoderType.CLIP_VIT, 336, 14, 24, 16, 1024, 4096, 4096, True)

    @classmethod
    def siglip_so14_224(cls) -> "VisionConfig":
        """SigLIP So400m/14 at 224 px (PaliGemma 3B): 256 patches, no CLS."""
        return cls(VisionEncoderType.SIGLIP, 224, 14, 27, 16, 1152, 4304, 2048, False)

    @classmethod
    def siglip2_896(cls) -> "VisionConfig":
        """SigLIP 2 at 896 px (Gemma 3 vision): 3136 patches."""
        return cls(VisionEncoderType.SIGLIP, 896, 16, 27, 16, 1152, 4304, 3072, False)

    @classmethod
    def tiny(cls, proj_dim: int = 256) -> "VisionConfig":
        return cls(VisionEncoderType.CLIP_VIT, 32, 8, 2, 4, 64, 128, proj_dim, True)


_CLIP_MEAN = (0.48145466, 0.4578275, 0.40821073)
_CLIP_STD = (0.26862954, 0.26130258, 0.27577711)


def normalize_image(image: torch.Tensor, use_siglip: bool) -> torch.Tensor:
    """[B, 3, H, W] in [0, 1] -> zero-mean unit-variance per channel (SigLIP: 0.5 / 0.5,
    CLIP: ImageNet statistics)."""
    mean = (0.5, 0.5, 0.5) if use_siglip else _CLIP_MEAN
    std = (0.5, 0.5, 0.5) if use_siglip else _CLIP_STD
    m = torch.tensor(mean, dtype=image.dtype, device=image.device).view(1, 3, 1, 1)
    s = torch.tensor(std, dtype=image.dtype, device=image.device).view(1, 3, 1, 1)
    return (image - m) / s


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    return 0.5 * x * (1.0 + torch.tanh(math.sqrt(2.0 / math.pi) * (x + 0.044715 * x * x * x)))


@dataclass
class VitLayer:
    ln1_w: torch.Tensor
    ln1_b: torch.Tensor | None
    wq: torch.Tensor
    wk: torch.Tensor
    wv: torch.Tensor
    wo: torch.Tensor
    ln2_w: torch.Tensor
    ln2_b: torch.Tensor | None
    fc1: torch.Tensor
    fc2: torch.Tensor
    bq: torch.Tensor | None = None
    bk: torch.Tensor | None = None
    bv: torch.Tensor | None = None
    bo: torch.Tensor | None = None
    b1: torch.Tensor | None = None
    b2: torch.Tensor | None = None


class VisionEncoder:
    """Weights: ``patch_w`` [hidden, 3, p, p] (+ bias), ``pos`` [1, patches (+1), hidden],
    optional ``cls`` [1, 1, hidden], layers, optional post-LN and projection [proj, hidden]."""

    eps = 1e-6

    def __init__(self, cfg: VisionConfig, patch_w, patch_b, pos, cls, layers, post_w=None, post_b=None,
                 proj=None, proj_b=None):
        self.cfg = cfg
        self.patch_w, self.patch_b, self.pos, self.cls = patch_w, patch_b, pos, cls
        self.layers = layers
        self.post_w, self.post_b, self.proj, self.proj_b = post_w, post_b, proj, proj_b

    @classmethod
    def random(cls, cfg: VisionConfig, device="cpu", dtype=torch.float32, seed: int = 0, std: float = 0.02):
        g = torch.Generator().manual_seed(seed)

        def r(*shape):
            return (torch.randn(*shape, generator=g) * std).to(device=device, dtype=dtype)

        def ones(n):
            return torch.ones(n, device=device, dtype=dtype)
        H, M, p = cfg.hidden_dim, cfg.mlp_dim, cfg.patch_size
        n_tok = cfg.num_patches + (1 if cfg.use_cls_token else 0)
        layers = [VitLayer(ones(H), r(H), r(H, H), r(H, H), r(H, H), r(H, H), ones(H), r(H), r(M, H), r(H, M),
                           r(H), r(H), r(H), r(H), r(M), r(H)) for _ in range(cfg.n_layers)]
        return cls(cfg, r(H, 3, p, p), r(H), r(1, n_tok, H), r(1, 1, H) if cfg.use_cls_token else None, layers,
                   ones(H), r(H), r(cfg.proj_dim, H), r(cfg.proj_dim))

    # ------------------------------------------------------------------ pieces
    def patch_embed(self, image: torch.Tensor) -> torch.Tensor:
        """[B, 3, H, W] -> [B, patches, hidden]: non-overlapping p x p patches flattened in
        (channel, row, column) order times the patch weight (a stride-p convolution)."""
        B, C, Hh, Ww = image.shape
        p = self.cfg.patch_size
        nh, nw = Hh // p, Ww // p
        x = image[:, :, : nh * p, : nw * p].reshape(B, C, nh, p, nw, p).permute(0, 2, 4, 1, 3, 5)
        x = x.reshape(B, nh * nw, C * p * p)
        out = x @ self.patch_w.reshape(self.patch_w.shape[0], -1).t()
        return out + self.patch_b if self.patch_b is not None else out

    def _ln(self, x, w, b):
        return F.layer_norm(x, (x.shape[-1],), w, b, self.eps)

    def _attn(self, x: torch.Tensor, L: VitLayer) -> torch.Tensor:
        B, S, Hd = x.shape
        nh = self.cfg.n_heads
        d = Hd // nh

        def proj(w, b):
            y = x @ w.t()
            return (y + b if b is not None else y).reshape(B, S, nh, d).transpose(1, 2)
        q, k, v = proj(L.wq, L.bq), proj(L.wk, L.bk), proj(L.wv, L.bv)
        ctx = F.scaled_dot_product_attention(q, k, v)        # bidirectional
        ctx = ctx.transpose(1, 2).reshape(B, S, Hd)
        o = ctx @ L.wo.t()
        return o + L.bo if L.bo is not None else o

    def layer_forward(self, x: torch.Tensor, L: VitLayer) -> torch.Tensor:
        x = x + self._attn(self._ln(x, L.ln1_w, L.ln1_b), L)
        h = self._ln(x, L.ln2_w, L.ln2_b) @ L.fc1.t()
        if L.b1 is not None:
            h = h + L.b1
        h = gelu_tanh(h) @ L.fc2.t()
        if L.b2 is not None:
            h = h + L.b2
        return x + h

    # ------------------------------------------------------------------ full encoder
    @torch.no_grad()
    def encode(self, image: torch.Tensor, normalize: bool = True) -> torch.Tensor:
        """[B, 3, H, W] in [0, 1] -> visual tokens [B, patches, proj_dim]."""
        cfg = self.cfg
        img = image.to(self.patch_w.dtype)
        if normalize:
            img = normalize_image(img, cfg.encoder_type == VisionEncoderType.SIGLIP)
        x = self.patch_embed(img)
        if self.cls is not None:
            x = torch.cat([self.cls.expand(x.shape[0], 1, -1), x], 1)
        x = x + self.pos
        for L in self.layers:
            x = self.layer_forward(x, L)
        if self.post_w is not None:
            x = self._ln(x, self.post_w, self.post_b)
        if cfg.use_cls_token:
            x = x[:, 1:1 + cfg.num_patches]
        if self.proj is not None:
            x = x @ self.proj.t()
            if self.proj_b is not None:
                x = x + self.proj_b
        return x


def image_prompt_hidden(token_embeddings: torch.Tensor, ids: list[int], image_tokens: torch.Tensor,
                        image_token_id: int) -> torch.Tensor:
    """Token embeddings [T, H] of a prompt with each run of ``image_token_id`` placeholders
    replaced, in order, by the rows of ``image_tokens`` [N, H] (LLaVA-style splicing). The
    number of placeholders must equal N."""
    pos = [i for i, t in enumerate(ids) if t == image_token_id]
    if len(pos) != image_tokens.shape[0]:
        raise ValueError(f"{len(pos)} image placeholders for {image_tokens.shape[0]} image tokens")
    out = token_embeddings.clone()
    if pos:
        out[torch.tensor(pos, device=out.device)] = image_tokens.to(out.dtype)
    return out
