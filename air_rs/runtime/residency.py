"""Residency planning: which layers (and MoE experts) stay in device memory and which stream
from pinned host memory (reference ``src/residency.rs``: GpuProfile, ModelBudget,
compute_residency -> ResidencyPlan with FullPin / SelfSpeculative / FullStream strategies).

``plan_model`` turns a ``ModelConfig`` and a weight format into the builder options:
everything resident when the weights, the KV hot tier and the workspace fit under the VRAM
cap (the normal case on a 180 GB B200, up to ~70B at 4 bits); otherwise dense models stream
layers through ``stream_slots`` device slots (S.L.I.P.), and MoE models keep the dense parts
resident and serve experts through an LRU expert cache sized to the room left.
"""
from __future__ import annotations

import enum
from dataclasses import dataclass

from ..gguf import BLOCK_GEOMETRY, GGMLType
from . import vram_guard

KV_HOT_TIER_MB = 1500.0
APPLE_PIN_BUDGET_RATIO = 0.30


@dataclass
class GpuProfile:
    name: str
    total_memory_mb: float
    unified_memory: bool = False
    pin_budget_ratio: float = 1.0
    compute_time_ms: float = 70.0      # one full-model forward at batch 1 (drafting estimate)

    @classmethod
    def b200(cls) -> "GpuProfile":
        return cls("NVIDIA B200", 183_359.0, False, 1.0, 2.1)

    @classmethod
    def rtx_4090(cls) -> "GpuProfile":
        return cls("NVIDIA RTX 4090", 24_576.0, False, 1.0, 70.0)

    @classmethod
    def rtx_3060(cls) -> "GpuProfile":
        return cls("NVIDIA RTX 3060", 12_288.0, False, 1.0, 72.0)

    @classmethod
    def apple_m3_pro(cls) -> "GpuProfile":
        return cls("Apple M3 Pro", 18_432.0, True, APPLE_PIN_BUDGET_RATIO, 50.0)

    @classmethod
    def custom(cls, name: str, total_memory_mb: float, unified: bool, compute_time_ms: float) -> "GpuProfile":
        return cls(name, total_memory_mb, unified, APPLE_PIN_BUDGET_RATIO if unified else 1.0, compute_time_ms)

    @classmethod
    def from_device(cls, device=0) -> "GpuProfile":
        import torch
        p = torch.cuda.get_device_properties(device)
        return cls(p.name, p.total_memory / 2**20, False, 1.0, 70.0)

    def available_memory_mb(self) -> float:
        return self.total_memory_mb * self.pin_budget_ratio


@dataclass
class ModelBudget:
    n_layers: int
    layer_size_mb: float
    kv_hot_tier_mb: float = KV_HOT_TIER_MB
    pipeline_buffer_mb: float | None = None

    def __post_init__(self):
        if self.pipeline_buffer_mb is None:
            self.pipeline_buffer_mb = 2 * self.layer_size_mb     # two streaming slots

    @classmethod
    def llama_70b_q4(cls) -> "ModelBudget":
        return cls(80, 531.0, KV_HOT_TIER_MB, 1062.0)

    def overhead_mb(self) -> float:
        return self.kv_hot_tier_mb + self.pipeline_buffer_mb


class ResidencyStrategy(str, enum.Enum):
    FULL_PIN = "full_pin"
    SELF_SPECULATIVE = "self_speculative"
    FULL_STREAM = "full_stream"


@dataclass
class ResidencyPlan:
    gpu_name: str
    n_resident: int
    n_layers: int
    full_pin: bool
    available_for_layers_mb: float
    layer_size_mb: float
    draft_time_ms: float
    full_compute_ms: float
    streaming_layers: int
    strategy: ResidencyStrategy

    def estimated_ttft_ms(self) -> float:
        return self.draft_time_ms if self.strategy == ResidencyStrategy.SELF_SPECULATIVE else self.full_compute_ms

    def pinned_vram_mb(self) -> float:
        return self.n_resident * self.layer_size_mb


def compute_residency(gpu: GpuProfile, model: ModelBudget) -> ResidencyPlan:
    """Layers that fit after the KV hot tier and pipeline buffers; a plan keeping >= 3 layers
    resident can self-draft from them."""
    avail = max(0.0, gpu.available_memory_mb() - model.overhead_mb())
    n_res = min(int(avail // model.layer_size_mb) if model.layer_size_mb > 0 else model.n_layers, model.n_layers)
    full = n_res >= model.n_layers
    draft = gpu.compute_time_ms * n_res / model.n_layers if model.n_layers else 0.0
    strat = (ResidencyStrategy.FULL_PIN if full else
             ResidencyStrategy.SELF_SPECULATIVE if n_res >= 3 else ResidencyStrategy.FULL_STREAM)
    return ResidencyPlan(gpu.name, n_res, model.n_layers, full, avail, model.layer_size_mb, draft,
                         gpu.compute_time_ms, model.n_layers - n_res, strat)


def bytes_per_weight(qtype: GGMLType) -> float:
    qtype = GGMLType(qtype)
    if qtype == GGMLType.F32:
        return 4.0
    if qtype in (GGMLType.F16, GGMLType.BF16):
        return 2.0
    per, nb = BLOCK_GEOMETRY[qtype]
    return nb / per


@dataclass
class BuildPlan:
    resident: bool
    stream_slots: int
    expert_slots: int | None
    weights_mb: float
    dense_mb: float
    cap_mb: float
    note: str
    resident_layers: int = 0          # streamed models: leading layers kept on the device


def plan_model(cfg, qtype: GGMLType, total_memory_mb: float, kv_mb: float = KV_HOT_TIER_MB,
               workspace_mb: float = 2048.0, cap_fraction: float | None = None) -> BuildPlan:
    """Builder options for ``cfg`` stored as ``qtype`` on a device of ``total_memory_mb``."""
    bpw = bytes_per_weight(qtype)
    H, V, L = cfg.hidden_dim, cfg.vocab_size, cfg.n_layers
    attn = (cfg.q_dim * H * 2 + cfg.kv_dim * H * 2) * bpw
    ffn_one = 3 * H * cfg.intermediate_dim * bpw
    n_exp = max(1, cfg.n_experts)
    dense = (2 * V * H * bpw + L * attn) / 2**20
    experts = L * ffn_one * n_exp / 2**20
    total = dense + experts
    cap = total_memory_mb * (cap_fraction or vram_guard.default_fraction())
    room = cap - kv_mb - workspace_mb
    if total <= room:
        return BuildPlan(True, 2, None, total, dense, cap, "all weights resident")
    if cfg.n_experts:
        per_expert = ffn_one / 2**20
        slots = int((room - dense) // per_expert)
        if slots >= max(cfg.moe_top_k, 1):
            return BuildPlan(True, 2, slots, total, dense, cap,
                             f"dense layers resident, {slots} of {L * n_exp} experts in device slots")
    layer = (attn + ffn_one * n_exp) / 2**20
    fit = int((room - 2 * V * H * bpw / 2**20) // max(layer, 1e-9))     # layers that fit on the device
    slots = 2
    keep = max(0, min(L - 1, fit - slots))
    return BuildPlan(False, slots, None, total, dense, cap,
                     f"{keep} layers resident, {L - keep} streamed through {slots} device slots", keep)
