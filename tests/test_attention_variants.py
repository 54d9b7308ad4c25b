"""FP4 micro-scaled attention, linear attention, gated attention output (reference
src/ops.rs:1700-2060 tests)."""
import torch

from air_rs.models.archs import attention_variants as A


def test_fp4_quantize_values_and_scale():
    x = torch.tensor([6.0, -3.0, 1.2, 0.2] + [0.0] * 12)
    q, s = A.fp4_quantize_blocked(x)
    assert s.tolist() == [1.0]
    assert q[:4].tolist() == [6.0, -3.0, 1.0, 0.0]
    y = torch.randn(5, 37)
    qy, sy = A.fp4_quantize_blocked(y)
    assert sy.numel() == (5 * 37 + 15) // 16
    # every value is sign * E2M1 level * its block's scale
    lv = (qy.reshape(-1).abs() / sy.repeat_interleave(16)[: 5 * 37])
    assert bool(torch.isclose(lv[..., None], A.FP4_VALUES).any(-1).all())


def test_fp4_attention_close_to_softmax():
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(1, 12, 4, 32, generator=g) * 0.5, torch.randn(1, 12, 2, 32, generator=g) * 0.5,
               torch.randn(1, 12, 2, 32, generator=g))
    ref = A.gqa_attention(q, k, v)
    out = A.fp4_attention(q, k, v)
    assert float((out - ref).abs().max()) < 0.35 and float((out - ref).abs().mean()) < 0.08


def test_linear_attention_matches_quadratic_form():
    g = torch.Generator().manual_seed(1)
    B, S, H, Hk, D = 2, 9, 4, 2, 8
    q, k, v = torch.randn(B, S, H, D, generator=g), torch.randn(B, S, Hk, D, generator=g), torch.randn(B, S, Hk, D, generator=g)
    out = A.linear_attention(q, k, v)
    pq, pk = A.phi_elu(q), A.phi_elu(k).repeat_interleave(2, 2)
    vv = v.repeat_interleave(2, 2)
    w = torch.einsum("bihd,bjhd->bhij", pq, pk).tril()
    ref = torch.einsum("bhij,bjhd->bihd", w, vv) / w.sum(-1).transpose(1, 2)[..., None]
    torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-5)
    # decode step against the last row of a longer context
    torch.testing.assert_close(A.linear_attention(q[:, -1:], k, v), out[:, -1:], rtol=1e-4, atol=1e-5)


def test_gated_output():
    a = torch.ones(1, 2, 3, 4)
    x = torch.zeros(1, 2, 12)
    x[..., :4] = 100.0
    x[..., 4:8] = -100.0
    o = A.gated_attention_output(a, x)
    assert torch.allclose(o[..., 0, :], torch.ones(1, 2, 4)) and float(o[..., 1, :].abs().max()) < 1e-6
    assert torch.allclose(o[..., 2, :], torch.full((1, 2, 4), 0.5))
    w = torch.zeros(3, 12)
    assert torch.allclose(A.gated_attention_output(a, x, w), a * 0.5)
