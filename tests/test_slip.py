"""S.L.I.P. layer streaming: host-resident layers streamed through device slots must give
the same tokens as the resident model, with copies overlapped by compute."""
import pytest
import torch

from air_rs.gguf import GGMLType
from air_rs.models.config import ModelConfig
from air_rs.models.random_init import random_tensors

pytestmark = pytest.mark.gpu


def test_streaming_matches_resident_and_overlaps():
    from air_rs.runtime.builder import build_runner
    from air_rs.runtime.engine import Engine, SamplingParams
    cfg = ModelConfig(n_layers=6, n_heads=8, n_kv_heads=2, hidden_dim=1024, intermediate_dim=2816,
                      vocab_size=4096, head_dim=128)
    recs = list(random_tensors(cfg, GGMLType.Q4_K, seed=0, device="cpu"))
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, cfg.vocab_size, (int(n),), generator=g).tolist() for n in (30, 12, 51)]
    sp = SamplingParams(max_tokens=16, temperature=0.0, repetition_penalty=1.0, ignore_eos=True)
    outs = []
    for resident in (True, False):
        rn = build_runner(cfg, iter(recs), device="cuda", max_batch=8, max_model_len=256, num_blocks=128,
                          resident=resident)
        rn._fused_ok = False        # same (separate-norm) decode chain as the streamed runner
        eng = Engine(cfg, rn, max_batch=8)
        outs.append(eng.generate_ids(prompts, sp))
        if not resident:
            assert rn.w.layers[0].wqkv.data.device.type == "cpu" and rn.w.layers[0].wqkv.data.is_pinned()
            st = rn.streamer.collect()
            per_layer = sum(t.numel() * t.element_size() for t in rn.streamer.slot_tensors[0])
            assert st.layers_loaded >= cfg.n_layers and st.bytes_h2d == st.layers_loaded * per_layer
            assert st.copy_ms > 0 and st.compute_ms > 0
            assert st.underruns >= 0 and st.stall_ms >= 0.0
    assert outs[0] == outs[1]


def test_partial_residency_matches_resident():
    """The first layers kept on the device, the rest streamed: same tokens, fewer copies."""
    from air_rs.runtime.builder import build_runner
    from air_rs.runtime.engine import Engine, SamplingParams
    cfg = ModelConfig(n_layers=6, n_heads=8, n_kv_heads=2, hidden_dim=1024, intermediate_dim=2816,
                      vocab_size=4096, head_dim=128)
    recs = list(random_tensors(cfg, GGMLType.Q4_K, seed=0, device="cpu"))
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, cfg.vocab_size, (int(n),), generator=g).tolist() for n in (25, 8)]
    sp = SamplingParams(max_tokens=10, temperature=0.0, repetition_penalty=1.0, ignore_eos=True)
    outs = []
    for kw in (dict(resident=True), dict(resident=False, resident_layers=3)):
        rn = build_runner(cfg, iter(recs), device="cuda", max_batch=8, max_model_len=256, num_blocks=128, **kw)
        rn._fused_ok = False
        outs.append(Engine(cfg, rn, max_batch=8).generate_ids(prompts, sp))
        if not kw["resident"]:
            st = rn.streamer.collect()
            assert sorted(rn.streamer.resident) == [0, 1, 2] and rn.streamer.streamed == [3, 4, 5]
            per_layer = sum(t.numel() * t.element_size() for t in rn.streamer.slot_tensors[0])
            assert st.bytes_h2d == st.layers_loaded * per_layer
    assert outs[0] == outs[1]
