"""Model hyperparameters from GGUF metadata.

Key names and defaults follow the reference (``src/model.rs:82-243``,
``src/model_variant.rs:41-189``): ``{arch}.block_count`` (32), ``.attention.head_count``
(32), ``.attention.head_count_kv`` (= heads), ``.embedding_length`` (4096),
``.feed_forward_length`` (11008), ``.vocab_size`` (or the tokenizer length, 32000),
``.rope.freq_base`` (500000 llama / 1e6 mistral,qwen2 / 1e4 other), ``.context_length``
(4096), ``.attention.layer_norm_rms_epsilon`` (1e-5), ``.attention.key_length``
(hidden/heads), ``.expert_count``/``.expert_used_count`` (0), ``.eos_token_id`` (2).
Unlike the reference, an ``expert_count > 0`` Llama/Mistral file maps to a softmax-MoE FFN,
so Mixtral-style checkpoints load.
"""
from __future__ import annotations

import enum
from dataclasses import dataclass, field, asdict
from typing import Any


class ModelVariant(str, enum.Enum):
    LLAMA = "llama"
    MISTRAL = "mistral"
    PHI3 = "phi3"
    PHI4 = "phi4"
    QWEN2 = "qwen2"
    QWEN3_6 = "qwen3_6"
    GEMMA = "gemma"
    GEMMA4 = "gemma4"
    FALCON = "falcon"
    UNKNOWN = "unknown"

    @classmethod
    def from_arch(cls, arch: str) -> "ModelVariant":
        a = arch.lower()
        table = {
            "llama": cls.LLAMA, "mistral": cls.MISTRAL, "phi3": cls.PHI3, "phi": cls.PHI3,
            "phi4": cls.PHI4, "qwen2": cls.QWEN2, "qwen": cls.QWEN2,
            "qwen3_5": cls.QWEN3_6, "qwen3.5": cls.QWEN3_6, "qwen3_6": cls.QWEN3_6,
            "qwen3.6": cls.QWEN3_6, "qwen35": cls.QWEN3_6,
            "gemma": cls.GEMMA, "gemma2": cls.GEMMA, "gemma3": cls.GEMMA, "gemma4": cls.GEMMA4,
            "falcon": cls.FALCON, "rw": cls.FALCON,
        }
        return table.get(a, cls.UNKNOWN)


class NormType(str, enum.Enum):
    RMS = "rmsnorm"
    LAYER = "layernorm"
    GEMMA_RMS = "gemma_rmsnorm"


class FfnType(str, enum.Enum):
    SWIGLU = "swiglu"
    GEGLU = "geglu"
    DENSE = "dense_mlp"
    SIGMOID_MOE = "sigmoid_moe"
    SOFTMAX_MOE = "softmax_moe"


_ROPE_DEFAULT = {ModelVariant.LLAMA: 500000.0, ModelVariant.MISTRAL: 1000000.0,
                 ModelVariant.QWEN2: 1000000.0}


@dataclass
class ModelConfig:
    n_layers: int = 2
    n_heads: int = 4
    n_kv_heads: int = 2
    hidden_dim: int = 256
    intermediate_dim: int = 688
    vocab_size: int = 4096
    rope_theta: float = 10000.0
    context_length: int = 4096
    rms_norm_eps: float = 1e-5
    head_dim: int = 64
    arch: str = "llama"
    variant: ModelVariant = ModelVariant.LLAMA
    norm_type: NormType = NormType.RMS
    ffn_type: FfnType = FfnType.SWIGLU
    sliding_window: int | None = None
    partial_rope_factor: float | None = None
    n_experts: int = 0
    moe_top_k: int = 0
    eos_token_id: int = 2
    bos_token_id: int = 1
    extra: dict[str, Any] = field(default_factory=dict)
    # per-architecture tensor layout (reference src/model.rs:326-360, src/weight_streamer.rs:215-250):
    qkv_bias: bool = False        # blk.N.attn_{q,k,v}.bias (Qwen2)
    norm_bias: bool = False       # blk.N.{attn,ffn}_norm.bias, output_norm.bias (Falcon LayerNorm)
    fused_qkv: bool = False       # blk.N.attn_qkv.weight = [q; k; v] rows (Phi-3)
    fused_gate_up: bool = False   # blk.N.ffn_up.weight = [gate; up] rows, no ffn_gate (Phi-3)
    attn_softcap: float = 0.0     # {arch}.attn_logit_softcapping: scores -> c * tanh(s / c) (Gemma-2)

    def detect_layout(self, tensor_names) -> "ModelConfig":
        """Set the layout flags from a checkpoint's tensor names (biases and fused tensors are
        optional per file, so metadata alone does not say)."""
        names = set(tensor_names)
        self.qkv_bias = "blk.0.attn_q.bias" in names
        self.norm_bias = "blk.0.attn_norm.bias" in names
        self.fused_qkv = "blk.0.attn_qkv.weight" in names and "blk.0.attn_q.weight" not in names
        self.fused_gate_up = ("blk.0.ffn_gate.weight" not in names and "blk.0.ffn_up.weight" in names
                              and self.ffn_type in (FfnType.SWIGLU, FfnType.GEGLU))
        return self

    @property
    def q_dim(self) -> int:
        return self.n_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    def to_dict(self) -> dict:
        d = asdict(self)
        d["variant"] = self.variant.value
        d["norm_type"] = self.norm_type.value
        d["ffn_type"] = self.ffn_type.value
        return d

    @classmethod
    def from_gguf_metadata(cls, md: dict[str, Any]) -> "ModelConfig":
        arch = str(md.get("general.architecture", "llama"))
        variant = ModelVariant.from_arch(arch)

        def g(key, default):
            v = md.get(f"{arch}.{key}")
            return default if v is None else v

        n_layers = int(g("block_count", 32))
        n_heads = int(g("attention.head_count", 32))
        n_kv = int(g("attention.head_count_kv", n_heads))
        hidden = int(g("embedding_length", 4096))
        inter = int(g("feed_forward_length", 11008))
        vocab = md.get(f"{arch}.vocab_size")
        if vocab is None:
            toks = md.get("tokenizer.ggml.tokens")
            vocab = len(toks) if toks is not None else 32000
        rope = float(g("rope.freq_base", _ROPE_DEFAULT.get(variant, 10000.0)))
        ctx = int(g("context_length", 4096))
        eps = md.get(f"{arch}.attention.layer_norm_rms_epsilon",
                     md.get(f"{arch}.attention.layer_norm_epsilon", 1e-5))
        head_dim = int(g("attention.key_length", hidden // max(n_heads, 1))) or 128
        n_exp = int(g("expert_count", 0))
        top_k = int(g("expert_used_count", 0))
        eos = md.get(f"{arch}.eos_token_id", md.get("tokenizer.ggml.eos_token_id", 2))
        bos = md.get("tokenizer.ggml.bos_token_id", 1)
        norm = {ModelVariant.GEMMA: NormType.GEMMA_RMS, ModelVariant.GEMMA4: NormType.GEMMA_RMS,
                ModelVariant.FALCON: NormType.LAYER}.get(variant, NormType.RMS)
        if n_exp > 0:
            ffn = FfnType.SIGMOID_MOE if variant == ModelVariant.GEMMA4 else FfnType.SOFTMAX_MOE
        else:
            ffn = {ModelVariant.GEMMA: FfnType.GEGLU, ModelVariant.FALCON: FfnType.DENSE}.get(
                variant, FfnType.SWIGLU)
        sw = md.get(f"{arch}.attention.sliding_window")
        if sw is None and variant == ModelVariant.MISTRAL:
            sw = None
        prf = None
        if variant == ModelVariant.PHI3:
            rd = md.get(f"{arch}.rope.dimension_count")
            if rd:
                prf = float(rd) / head_dim
        extra = {}
        pattern = md.get(f"{arch}.attention.sliding_window_pattern")
        if sw and pattern and int(pattern) > 1:
            # local (sliding) layers with every pattern-th layer global, the last one included
            from .archs.hybrid import HybridAttentionRouter
            extra["attention_layout"] = HybridAttentionRouter.gemma4(
                n_layers, int(sw), int(pattern)).windows()
        return cls(attn_softcap=float(md.get(f"{arch}.attn_logit_softcapping", 0.0) or 0.0),
                   qkv_bias=variant == ModelVariant.QWEN2, norm_bias=variant == ModelVariant.FALCON,
                   fused_qkv=variant == ModelVariant.PHI3, fused_gate_up=variant == ModelVariant.PHI3,
                   n_layers=n_layers, n_heads=n_heads, n_kv_heads=n_kv, hidden_dim=hidden,
                   intermediate_dim=inter, vocab_size=int(vocab), rope_theta=rope,
                   context_length=ctx, rms_norm_eps=float(eps), head_dim=head_dim, arch=arch,
                   variant=variant, norm_type=norm, ffn_type=ffn,
                   sliding_window=int(sw) if sw else None, partial_rope_factor=prf,
                   n_experts=n_exp, moe_top_k=top_k, eos_token_id=int(eos), bos_token_id=int(bos),
                   extra=extra)

    def gguf_metadata(self) -> dict[str, Any]:
        a = self.arch
        md = {
            f"{a}.block_count": self.n_layers,
            f"{a}.attention.head_count": self.n_heads,
            f"{a}.attention.head_count_kv": self.n_kv_heads,
            f"{a}.embedding_length": self.hidden_dim,
            f"{a}.feed_forward_length": self.intermediate_dim,
            f"{a}.vocab_size": self.vocab_size,
            f"{a}.rope.freq_base": float(self.rope_theta),
            f"{a}.context_length": self.context_length,
            f"{a}.attention.layer_norm_rms_epsilon": float(self.rms_norm_eps),
            f"{a}.attention.key_length": self.head_dim,
            f"{a}.attention.value_length": self.head_dim,
            f"{a}.eos_token_id": self.eos_token_id,
        }
        if self.n_experts:
            md[f"{a}.expert_count"] = self.n_experts
            md[f"{a}.expert_used_count"] = self.moe_top_k
        if self.sliding_window:
            md[f"{a}.attention.sliding_window"] = self.sliding_window
        if self.attn_softcap > 0:
            md[f"{a}.attn_logit_softcapping"] = float(self.attn_softcap)
        return md


# Named benchmark shapes (from the benchmark configs).
def tiny_llama() -> ModelConfig:
    return ModelConfig(n_layers=2, n_heads=4, n_kv_heads=2, hidden_dim=256, intermediate_dim=688,
                       vocab_size=4096, rope_theta=10000.0, rms_norm_eps=1e-5, head_dim=64)


def llama3_8b() -> ModelConfig:
    return ModelConfig(n_layers=32, n_heads=32, n_kv_heads=8, hidden_dim=4096,
                       intermediate_dim=14336, vocab_size=128256, rope_theta=500000.0,
                       context_length=8192, head_dim=128, eos_token_id=128001, bos_token_id=128000)


def llama3_70b() -> ModelConfig:
    return ModelConfig(n_layers=80, n_heads=64, n_kv_heads=8, hidden_dim=8192,
                       intermediate_dim=28672, vocab_size=128256, rope_theta=500000.0,
                       context_length=8192, head_dim=128, eos_token_id=128001, bos_token_id=128000)


def mixtral_8x7b() -> ModelConfig:
    return ModelConfig(n_layers=32, n_heads=32, n_kv_heads=8, hidden_dim=4096,
                       intermediate_dim=14336, vocab_size=32000, rope_theta=1000000.0,
                       context_length=32768, head_dim=128, ffn_type=FfnType.SOFTMAX_MOE,
                       n_experts=8, moe_top_k=2)


def draft_1b() -> ModelConfig:
    return ModelConfig(n_layers=16, n_heads=32, n_kv_heads=8, hidden_dim=2048,
                       intermediate_dim=8192, vocab_size=128256, rope_theta=500000.0,
                       context_length=8192, head_dim=64, eos_token_id=128001, bos_token_id=128000)


def tiny_moe() -> ModelConfig:
    """Tiny Mixtral-style model (4 experts, top-2) for tests."""
    return ModelConfig(n_layers=2, n_heads=4, n_kv_heads=2, hidden_dim=256, intermediate_dim=256,
                       vocab_size=4096, rope_theta=10000.0, rms_norm_eps=1e-5, head_dim=64,
                       variant=ModelVariant.MISTRAL, n_experts=4, moe_top_k=2)


def tiny_variant(arch: str) -> ModelConfig:
    """Tiny model of an architecture variant (tests): qwen2 (q/k/v biases), gemma (Gemma
    RMSNorm + GeGLU), falcon (LayerNorm with biases + dense GELU MLP), phi3 (fused attn_qkv and
    gate|up tensors)."""
    v = ModelVariant.from_arch(arch)
    c = tiny_llama()
    c.arch, c.variant = arch, v
    c.intermediate_dim = 512
    if v == ModelVariant.QWEN2:
        c.qkv_bias = True
    elif v == ModelVariant.GEMMA:
        c.norm_type, c.ffn_type = NormType.GEMMA_RMS, FfnType.GEGLU
        c.attn_softcap = 50.0
    elif v == ModelVariant.FALCON:
        c.norm_type, c.ffn_type, c.norm_bias = NormType.LAYER, FfnType.DENSE, True
    elif v == ModelVariant.PHI3:
        c.fused_qkv = c.fused_gate_up = True
    return c


PRESETS = {"tiny": tiny_llama, "tiny-qwen2": lambda: tiny_variant("qwen2"),
           "tiny-gemma": lambda: tiny_variant("gemma"), "tiny-falcon": lambda: tiny_variant("falcon"),
           "tiny-phi3": lambda: tiny_variant("phi3"), "tiny-moe": tiny_moe, "llama3-8b": llama3_8b, "llama3-70b": llama3_70b,
           "mixtral-8x7b": mixtral_8x7b, "draft-1b": draft_1b}
