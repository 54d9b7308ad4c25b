"""Per-layer attention layouts (reference src/attention_backend.rs tests): router layouts,
GGUF sliding-window patterns, and sliding / global interleaving in the oracle and the GPU
runner."""
import pytest
import torch

from air_rs.models.archs.hybrid import AttentionBackend, Backend, HybridAttentionRouter, layout_for_config, with_layout
from air_rs.models.config import ModelConfig, tiny_llama


def test_router_layouts():
    q = HybridAttentionRouter.qwen3_6_27b()
    assert q.n_layers() == 64 and q.count(AttentionBackend.delta_net()) == 48
    assert q.backend_for_layer(3) == AttentionBackend.softmax() and q.backend_for_layer(0).is_recurrent
    assert HybridAttentionRouter.qwen3_6_35b_a3b().n_layers() == 96
    g = HybridAttentionRouter.gemma4(12, 512, 6)
    kinds = [b.kind for b in g.layout()]
    assert kinds[5] == Backend.GLOBAL_FULL and kinds[11] == Backend.GLOBAL_FULL
    assert kinds.count(Backend.GLOBAL_FULL) == 2 and g.backend_for_layer(0).window == 512
    assert g.windows() == [512] * 5 + [0] + [512] * 5 + [0]
    d = HybridAttentionRouter.deepseek_v2(4)
    assert all(b.is_mla for b in d.layout())
    with pytest.raises(NotImplementedError):
        d.windows()
    with pytest.raises(ValueError):
        HybridAttentionRouter([])
    assert str(AttentionBackend.sliding(8)) == "SlidingWindow(w=8)" and AttentionBackend.mla().name == "mla"


def test_layout_from_config_and_metadata():
    cfg = tiny_llama()
    assert layout_for_config(cfg).windows() == [0, 0]
    md = cfg.gguf_metadata()
    md["llama.attention.sliding_window"] = 64
    md["llama.attention.sliding_window_pattern"] = 2
    c2 = ModelConfig.from_gguf_metadata(md)
    assert layout_for_config(c2).windows() == [64, 0]
    c3 = with_layout(cfg, HybridAttentionRouter([AttentionBackend.sliding(4), AttentionBackend.global_full()]))
    assert layout_for_config(c3).windows() == [4, 0]


def test_oracle_sliding_layer_ignores_old_tokens():
    """With a 4-token window in every layer, the logits of the last token depend only on the
    last 4 * n_layers positions' reach; changing the first token of a long prompt leaves them
    unchanged once it is out of every layer's receptive field."""
    from air_rs.gguf import GGMLType
    from air_rs.models.random_init import random_tensors
    from air_rs.models.reference import OracleModel
    cfg = with_layout(tiny_llama(), HybridAttentionRouter.uniform(2, AttentionBackend.sliding(4)))
    recs = list(random_tensors(cfg, GGMLType.Q8_0, seed=0, device="cpu"))
    m = OracleModel(cfg, {n: (r, q, s) for n, r, q, s in recs})
    p = list(range(5, 30))
    a = m.forward(p, 0)
    m.reset()
    b = m.forward([7] + p[1:], 0)
    m.reset()
    assert torch.allclose(a, b)
    full = with_layout(tiny_llama(), HybridAttentionRouter.uniform(2, AttentionBackend.global_full()))
    mf = OracleModel(full, {n: (r, q, s) for n, r, q, s in recs})
    c = mf.forward(p, 0)
    mf.reset()
    d = mf.forward([7] + p[1:], 0)
    assert not torch.allclose(c, d)


@pytest.mark.gpu
def test_gpu_runner_interleaved_windows_match_oracle():
    from air_rs.gguf import GGMLType
    from air_rs.models.random_init import random_tensors
    from air_rs.models.reference import OracleModel
    from air_rs.runtime.builder import build_runner
    from air_rs.runtime.engine import Engine, SamplingParams
    from test_engine_gpu import _check_near_argmax
    base = ModelConfig(n_layers=4, n_heads=4, n_kv_heads=2, hidden_dim=512, intermediate_dim=1536,
                       vocab_size=4096, head_dim=128)
    cfg = with_layout(base, HybridAttentionRouter.gemma4(4, 16, 2))
    recs = list(random_tensors(cfg, GGMLType.Q4_K, seed=5, device="cpu"))
    oracle = OracleModel(cfg, {n: (r, q, s) for n, r, q, s in recs})
    rn = build_runner(cfg, iter(recs), device="cuda", max_batch=8, max_model_len=256, num_blocks=128)
    assert rn.layer_window == [16, 0, 16, 0]
    eng = Engine(cfg, rn, max_batch=8)
    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (40, 9, 70)]
    outs = eng.generate_ids(prompts, SamplingParams(max_tokens=12, temperature=0.0, ignore_eos=True))
    for p, o in zip(prompts, outs):
        _check_near_argmax(oracle, [cfg.bos_token_id] + p, o)
    rn.check_errors()
