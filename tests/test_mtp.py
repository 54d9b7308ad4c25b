"""Multi-token prediction heads (reference src/multi_token.rs tests)."""
import pytest
import torch

from air_rs.spec.mtp import MtpConfig, MtpHead, MtpHeads, mtp_forward_all, mtp_speculative_draft, rms_norm


def test_config_and_norm():
    c = MtpConfig.deepseek_v3()
    assert c.n_extra_heads == 1 and c.vocab_size == 102400 and c.hidden_dim == 7168 and c.enabled_at_inference
    v = rms_norm(torch.tensor([[1.0, 2.0, 4.0]]), torch.ones(3))
    assert abs(float(v[0, 0]) - 1 / (7 ** 0.5)) < 1e-4


def test_forward_all_and_draft():
    H, V = 16, 40
    lm = torch.randn(V, H)
    heads = MtpHeads.random(H, 2, seed=1)
    h = torch.randn(3, H)
    main, extra = mtp_forward_all(h, lambda x: x @ lm.t(), heads)
    assert main.shape == (3, V) and len(extra) == 2 and extra[0].shape == (3, V)
    ref = (rms_norm(h, heads.heads[0].norm_weight) @ heads.heads[0].proj.t()) @ lm.t()
    torch.testing.assert_close(extra[0], ref)
    m, d = mtp_speculative_draft(main, extra)
    assert m == int(main[-1].argmax()) and d == int(extra[0][-1].argmax())
    own = MtpHead(torch.ones(H), torch.eye(H), torch.zeros(H), lm_head=torch.randn(V, H))
    assert own.forward(h).shape == (3, V)
    off = MtpHeads(heads.heads, MtpConfig(2, V, H, enabled_at_inference=False))
    assert off.n_heads == 0 and off.logits(h, None) == []


@pytest.mark.gpu
def test_mtp_heads_draft_through_target_verification():
    from air_rs.runtime.builder import random_engine
    from air_rs.spec.medusa import MedusaDecoder
    from test_spec import _greedy_margin
    tgt = random_engine("tiny", seed=1, device="cuda:0", max_batch=8, max_model_len=512)
    heads = MtpHeads.random(tgt.runner.H, 2, device="cuda:0")
    dec = MedusaDecoder(tgt, heads, top_c=2, eos_id=-1)
    prompt = [3, 17, 29, 41, 5]
    outs, stats = dec.generate_batch([prompt], max_tokens=20)
    gap, spread = _greedy_margin(tgt, prompt, outs[0])
    assert len(outs[0]) == 20 and (gap <= 0.05 * spread).all()
    assert stats.drafted > 0
