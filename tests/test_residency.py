"""Residency planning (reference src/residency.rs tests) and builder plans for B200."""
from air_rs.gguf import GGMLType
from air_rs.models.config import PRESETS
from air_rs.runtime.residency import (GpuProfile, ModelBudget, ResidencyStrategy, bytes_per_weight,
                                      compute_residency, plan_model)


def test_compute_residency_strategies():
    p = compute_residency(GpuProfile.rtx_4090(), ModelBudget.llama_70b_q4())
    assert p.strategy == ResidencyStrategy.SELF_SPECULATIVE and p.n_resident == int((24576 - 2562) // 531)
    assert p.streaming_layers == 80 - p.n_resident and abs(p.pinned_vram_mb() - p.n_resident * 531) < 1e-9
    assert abs(p.estimated_ttft_ms() - 70.0 * p.n_resident / 80) < 1e-9
    full = compute_residency(GpuProfile.b200(), ModelBudget.llama_70b_q4())
    assert full.full_pin and full.strategy == ResidencyStrategy.FULL_PIN and full.estimated_ttft_ms() == 2.1
    tiny = compute_residency(GpuProfile.custom("x", 2000, False, 90), ModelBudget.llama_70b_q4())
    assert tiny.strategy == ResidencyStrategy.FULL_STREAM and tiny.n_resident == 0
    assert GpuProfile.apple_m3_pro().available_memory_mb() == 18432 * 0.30


def test_bytes_per_weight():
    assert bytes_per_weight(GGMLType.Q4_K) == 144 / 256 and bytes_per_weight(GGMLType.Q8_0) == 34 / 32
    assert bytes_per_weight(GGMLType.BF16) == 2.0


def test_plan_model_b200():
    b200 = GpuProfile.b200().total_memory_mb
    p = plan_model(PRESETS["llama3-8b"](), GGMLType.Q4_K, b200)
    assert p.resident and p.expert_slots is None and 4000 < p.weights_mb < 6000
    p70 = plan_model(PRESETS["llama3-70b"](), GGMLType.Q4_K, b200)
    assert p70.resident                                   # ~40 GB at 4 bits
    small = plan_model(PRESETS["llama3-70b"](), GGMLType.Q4_K, 24576)
    assert not small.resident and small.stream_slots == 2 and 0 < small.resident_layers < 80
    moe = plan_model(PRESETS["mixtral-8x7b"](), GGMLType.Q8_0, 40960)
    assert moe.resident and moe.expert_slots is not None and moe.expert_slots >= 2
