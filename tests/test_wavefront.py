"""Wavefront policy and FFN sparsity predictors (reference ``src/wavefront.rs:264-340`` and
``src/sparsity_predictor.rs:294-341`` test scenarios), plus the predictor trained and applied
on the CPU oracle model's real FFN activations."""
import pytest
import torch

from air_rs.spec.wavefront import (CycleStats, LayerSparsityPredictor, SparseFFNHook, SparseWeightMask,
                                   SparsityConfig, SparsityPredictorBank, WavefrontConfig,
                                   WavefrontHealthMonitor, WavefrontSession, compute_union_mask)


def test_predict_returns_sorted_topk_indices():
    cfg = SparsityConfig(64, 256, 0.2)
    p = LayerSparsityPredictor(cfg, seed=1)
    idx = p.predict_active(torch.randn(64))
    assert idx.numel() == cfg.top_k() == 52
    assert torch.equal(idx, idx.sort().values) and idx.unique().numel() == idx.numel()
    batch = p.predict_active(torch.randn(5, 64))
    assert batch.shape == (5, 52) and (batch[:, 1:] > batch[:, :-1]).all()


def test_masks_union_and_density():
    d = SparseWeightMask.dense(100)
    assert d.n_active() == 100 and d.density() == 1.0 and d.bytes_saved(4096) == 0
    m = SparseWeightMask(torch.tensor([1, 5, 9]), 10)
    assert m.n_active() == 3 and abs(m.density() - 0.3) < 1e-9
    assert m.bytes_saved(8, bytes_per_weight=2.0, n_matrices=3) == 7 * 8 * 2 * 3
    u = compute_union_mask([[0, 2, 4], [2, 3], [99, -1, 4]], 10)
    assert u.active_indices.tolist() == [0, 2, 3, 4]
    assert compute_union_mask([], 7).n_active() == 7
    assert m.as_bool().tolist() == [i in (1, 5, 9) for i in range(10)]


def test_bank_predict_mask_and_reduction():
    cfg = SparsityConfig.for_model(32, 128)
    bank = SparsityPredictorBank(3, cfg)
    m = bank.predict_mask(torch.randn(32), 1)
    assert m.n_active() == cfg.top_k() and m.total_rows == 128
    wave = bank.predict_mask(torch.randn(4, 32), 2)          # union over a 4-token wavefront
    assert cfg.top_k() <= wave.n_active() <= 128
    assert abs(bank.bandwidth_reduction() - 5.0) < 1e-9
    z = LayerSparsityPredictor.zeros(cfg)
    assert z.accuracy_ema == 0.0 and torch.all(z.scores(torch.randn(32)) == 0.5)


def test_online_training_learns_a_planted_pattern():
    torch.manual_seed(0)
    H, I = 32, 96
    W_true = torch.randn(I, H)
    cfg = SparsityConfig(H, I, 0.25)
    p = LayerSparsityPredictor(cfg, seed=3)

    def batch():
        h = torch.randn(64, H)
        return h, torch.relu(h @ W_true.t()) * (torch.rand(64, I) > 0.3)

    h, a = batch()
    before = p.measure_accuracy(p.predict_active(h[0]), a[0])
    for _ in range(300):
        hb, ab = batch()
        p.update(hb, ab, lr=0.01)
    recalls = [p.measure_accuracy(p.predict_active(hb[i]), ab[i]) for hb, ab in [batch()] for i in range(16)]
    after = sum(recalls) / len(recalls)
    assert after > before + 0.2 and after > 0.45     # top 25% kept, ~35% active: ceiling ~0.7


def test_health_monitor_adapts_up_and_down():
    m = WavefrontHealthMonitor(8)
    for _ in range(6):
        m.update(8, 8)
    assert m.current_draft_size > 8 and m.mean_acceptance() == 1.0
    m = WavefrontHealthMonitor(8)
    for _ in range(6):
        m.update(1, 8)
    assert m.current_draft_size < 8
    m.update(3, 0)                           # nothing drafted: ignored
    assert len(m.window) == 6
    m = WavefrontHealthMonitor(1, min_draft_size=1)
    for _ in range(30):
        m.update(0, 4)
    assert m.current_draft_size == 1 and len(m.window) == 20


def test_cycle_stats_session_and_config():
    c = CycleStats(draft_ms=10, io_ms=20, verify_ms=70, tokens_accepted=5, tokens_drafted=8,
                   sparsity_density=0.25, bytes_saved=3_000_000)
    assert abs(c.effective_tps() - 50.0) < 1e-9 and "accept=5/8" in c.display()
    assert CycleStats().effective_tps() == 0.0
    s = WavefrontSession()
    s.record(c)
    s.record(c)
    assert s.total_tokens == 12 and s.total_cycles == 2 and s.total_bytes_saved == 6_000_000
    assert abs(s.overall_tps() - 60.0) < 1e-9 and abs(s.acceptance_rate() - 5 / 8) < 1e-9
    assert "12 tokens in 2 cycles" in s.summary() and s.speedup_estimate() == 6.0
    assert WavefrontConfig.disabled().draft_size == 1 and not WavefrontConfig.disabled().async_double_buffer
    a = WavefrontConfig.aggressive(32)
    assert a.draft_size == 32 and a.sparsity_fraction == 0.2 and not a.verbose


def _oracle():
    from air_rs.gguf import GGMLType, read_gguf
    from air_rs.models.config import tiny_llama
    from air_rs.models.random_init import write_random_gguf
    from air_rs.models.reference import OracleModel
    import tempfile, os
    d = tempfile.mkdtemp()
    p = os.path.join(d, "m.gguf")
    cfg = tiny_llama()
    write_random_gguf(p, cfg, GGMLType.Q8_0, seed=0)
    return cfg, OracleModel.from_gguf(read_gguf(p))


def test_oracle_hook_observes_and_masks_ffn():
    cfg, m = _oracle()
    ids = [5, 17, 33, 2, 9]
    dense = m.forward(ids, 0)
    m.reset()
    bank = SparsityPredictorBank(cfg.n_layers, SparsityConfig(cfg.hidden_dim, cfg.intermediate_dim, 1.0))
    hook = SparseFFNHook(bank, learn=True, mask=True)
    m.ffn_hook = hook
    full = m.forward(ids, 0)                         # fraction 1.0: every neuron kept
    assert torch.equal(full, dense)
    assert len(hook.recalls) == cfg.n_layers and all(r == 1.0 for r in hook.recalls)
    assert hook.densities == [1.0] * cfg.n_layers
    m.reset()
    bank.config.top_k_fraction = 0.25
    hook = SparseFFNHook(bank, learn=False, mask=True)
    m.ffn_hook = hook
    sparse = m.forward(ids, 0)
    assert torch.isfinite(sparse).all() and not torch.equal(sparse, dense)
    assert all(0.25 <= d <= 1.0 for d in hook.densities)
    m.ffn_hook = None
    m.reset()
    assert torch.equal(m.forward(ids, 0), dense)


def test_medusa_heads_manifest_sidecar(tmp_path):
    from air_rs.spec.medusa import MedusaHeads
    h = MedusaHeads(16, n_heads=11, device="cpu", seed=2)
    p = str(tmp_path / "heads.pt")
    man = h.save(p, fingerprint=b"\x07" * 32, target_name="llama-3-8b")
    assert man.endswith(".draft.json")
    back = MedusaHeads.load(p, device="cpu", fingerprint=b"\x07" * 32, hidden=16)
    assert back.n_heads == 11 and all(torch.equal(a[0], b[0]) and torch.equal(a[1], b[1]) for a, b in zip(h.W, back.W))   # head10 after head9
    with pytest.raises(ValueError, match="another target"):
        MedusaHeads.load(p, device="cpu", fingerprint=b"\x08" * 32)
    with pytest.raises(ValueError, match="not 32 x 32"):
        MedusaHeads.load(p, device="cpu", hidden=32)
    import json
    m = json.load(open(man))
    m["n_heads"] = 3
    json.dump(m, open(man, "w"))
    with pytest.raises(ValueError, match="manifest"):
        MedusaHeads.load(p, device="cpu")


def test_medusa_heads_math_and_gguf(tmp_path):
    """Residual SwiGLU block h + silu(h W1^T) * (h W2^T) (reference src/medusa_heads.rs:89-94),
    loaded from GGUF tensors mtp_head.{i}.weight0/weight1."""
    import torch.nn.functional as F
    from air_rs.gguf import GGMLType
    from air_rs.gguf.writer import GGUFWriter
    from air_rs.spec.medusa import MedusaHeads
    g = torch.Generator().manual_seed(5)
    pairs = [(torch.randn(16, 16, generator=g), torch.randn(16, 16, generator=g)) for _ in range(2)]
    p = str(tmp_path / "mtp.gguf")
    wr = GGUFWriter(p)
    for i, (a, b) in enumerate(pairs):
        wr.add_tensor(f"mtp_head.{i}.weight0", a.contiguous().view(torch.uint8).flatten(), (16, 16), GGMLType.F32)
        wr.add_tensor(f"mtp_head.{i}.weight1", b.contiguous().view(torch.uint8).flatten(), (16, 16), GGMLType.F32)
    wr.write()
    heads = MedusaHeads.load(p, device="cpu", hidden=16)
    assert heads.n_heads == 2
    h = torch.randn(3, 16, generator=g)
    for (a, b), t in zip(pairs, heads.hidden(h)):
        torch.testing.assert_close(t, h + F.silu(h @ a.t()) * (h @ b.t()))
    with pytest.raises(ValueError, match="requested"):
        MedusaHeads.from_gguf(p, n_heads=3, device="cpu")


def test_medusa_heads_bad_keys(tmp_path):
    from air_rs.spec.medusa import MedusaHeads
    p = str(tmp_path / "bad.pt")
    torch.save({"head_norm": torch.zeros(4)}, p)
    with pytest.raises(ValueError, match="unexpected key"):
        MedusaHeads.load(p, device="cpu")
