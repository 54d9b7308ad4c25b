"""Reference implementations of the other architectures (reference LIB modules mla.rs,
mamba.rs, rwkv.rs, gated_deltanet.rs, yarn.rs, gemma4.rs, ops.rs variants)."""
import math

import pytest

import torch

from air_rs.models.archs import gemma, mla, rope_ext as R, ssm

G = lambda s: torch.Generator().manual_seed(s)


def test_mla_absorbed_equals_explicit_and_cache_is_small():
    w = mla.MlaWeights.random()
    x = torch.randn(7, 64, generator=G(0))
    pos = torch.arange(7)
    torch.testing.assert_close(mla.mla_forward(w, x, pos), mla.mla_forward_absorbed(w, x, pos), rtol=1e-4, atol=1e-5)
    c, kr = mla.latent_cache(w, x, pos)
    assert c.shape[1] + kr.shape[1] == 20 < 2 * 4 * 8        # latent + shared rope key vs per-head K, V
    # decode step against the cache of the whole sequence
    full = mla.mla_forward(w, x, pos)
    last = mla.mla_forward_absorbed(w, x[-1:], pos[-1:], cache=(c, kr))
    torch.testing.assert_close(last, full[-1:], rtol=1e-4, atol=1e-5)


def test_mamba_scans_agree():
    L, d, n = 9, 6, 4
    g = G(1)
    u, delta = torch.randn(L, d, generator=g), torch.rand(L, d, generator=g) * 0.5
    A = -torch.rand(d, n, generator=g)
    B, C = torch.randn(L, n, generator=g), torch.randn(L, n, generator=g)
    D, z = torch.randn(d, generator=g), torch.randn(L, d, generator=g)
    torch.testing.assert_close(ssm.selective_scan_ref(u, delta, A, B, C, D, z),
                               ssm.selective_scan_parallel(u, delta, A, B, C, D, z), rtol=1e-4, atol=1e-5)
    y = ssm.ssd_mamba2_ref(torch.randn(5, 2, 3, generator=g), torch.rand(5, 2, generator=g), -torch.rand(2, generator=g),
                           torch.randn(5, 4, generator=g), torch.randn(5, 4, generator=g))
    assert y.shape == (5, 2, 3)


def test_rwkv4_recurrent_matches_definition():
    g = G(2)
    k, v = torch.randn(8, 5, generator=g), torch.randn(8, 5, generator=g)
    w, u = torch.rand(5, generator=g), torch.randn(5, generator=g)
    torch.testing.assert_close(ssm.wkv_rwkv4_recurrent(w, u, k, v), ssm.wkv_rwkv4_ref(w, u, k, v), rtol=1e-4, atol=1e-5)
    o = ssm.wkv_rwkv6_ref(torch.randn(6, 4, generator=g), torch.randn(6, 4, generator=g), torch.randn(6, 3, generator=g),
                          torch.rand(6, 4, generator=g), torch.randn(4, generator=g))
    assert o.shape == (6, 3)


def test_gated_delta_rule_chunked_and_state():
    g = G(3)
    L, dk, dv = 10, 4, 3
    k = torch.nn.functional.normalize(torch.randn(L, dk, generator=g), dim=-1)
    q, v = torch.randn(L, dk, generator=g), torch.randn(L, dv, generator=g)
    a, b = torch.rand(L, generator=g), torch.rand(L, generator=g)
    o1, s1 = ssm.gated_delta_rule_ref(q, k, v, a, b)
    o2, s2 = ssm.gated_delta_rule_chunked(q, k, v, a, b, chunk=3)
    torch.testing.assert_close(o1, o2)
    torch.testing.assert_close(s1, s2)
    # with alpha = beta = 1 the state stores v for k exactly (delta rule overwrite)
    k1 = torch.tensor([[1.0, 0, 0, 0]])
    _, s = ssm.gated_delta_rule_ref(k1, k1, torch.tensor([[2.0, 3.0, 4.0]]), torch.ones(1), torch.ones(1))
    torch.testing.assert_close(s @ k1[0], torch.tensor([2.0, 3.0, 4.0]))
    y = ssm.causal_conv1d(torch.eye(4), torch.tensor([[1.0, 2.0]] * 4))
    assert y[0].tolist() == [2.0, 0, 0, 0] and y[1].tolist() == [1.0, 2.0, 0, 0]


def test_rope_variants_and_yarn():
    f = R.inv_freq(8, 10000.0)
    x = torch.randn(3, 2, 8, generator=G(4))
    pos = torch.tensor([0, 5, 9])
    y = R.rope_neox(x, pos, f)
    torch.testing.assert_close(y.norm(dim=-1), x.norm(dim=-1))         # rotation preserves norm
    torch.testing.assert_close(R.rope_neox(x, pos, f, rot_dim=4)[..., 4:], x[..., 4:])
    torch.testing.assert_close(R.rope_interleaved(x, pos, f).norm(dim=-1), x.norm(dim=-1))
    s = R.llama3_scaled_freqs(R.inv_freq(128, 500000.0))
    base = R.inv_freq(128, 500000.0)
    assert torch.allclose(s[0], base[0]) and torch.allclose(s[-1], base[-1] / 8.0)
    yf = R.YarnFrequencies(128, 10000.0, 4.0, 4096)
    assert abs(yf.mscale - (0.1 * math.log(4) + 1)) < 1e-9
    assert torch.allclose(yf.freqs[0], R.inv_freq(128, 10000.0)[0])
    assert torch.allclose(yf.freqs[-1], R.inv_freq(128, 10000.0)[-1] / 4.0)
    assert torch.allclose(R.alibi_slopes(8), torch.tensor([2 ** -(i + 1) for i in range(8)]))
    assert R.alibi_slopes(12).numel() == 12
    pe = R.sinusoidal_positions(4, 6)
    assert pe[0, 0] == 0 and pe[0, 1] == 1


def test_gemma_ops():
    x = torch.randn(3, 16, generator=G(5))
    w = torch.zeros(16)
    torch.testing.assert_close(gemma.gemma_rms_norm(x, w), x / torch.sqrt((x * x).mean(-1, keepdim=True) + 1e-6))
    torch.testing.assert_close(gemma.gelu_tanh(x), torch.nn.functional.gelu(x, approximate="tanh"))
    assert float(gemma.softcap(torch.tensor(1e6), 30.0)) <= 30.0
    q = torch.randn(4, 2, 8, generator=G(6))
    o = gemma.softcapped_attention(q, q, q, cap=1e9)
    ref = torch.nn.functional.scaled_dot_product_attention(q.transpose(0, 1), q.transpose(0, 1), q.transpose(0, 1),
                                                           is_causal=True).transpose(0, 1)
    torch.testing.assert_close(o, ref, rtol=1e-4, atol=1e-5)
    ids, wt = gemma.sigmoid_moe_route(torch.tensor([[0.0, 3.0, -1.0, 2.0]]), 2)
    assert ids.tolist() == [[1, 3]] and abs(float(wt.sum()) - 1) < 1e-6
    eo = torch.arange(8.0).reshape(1, 4, 2)
    torch.testing.assert_close(gemma.moe_weighted_sum(eo, ids, wt), (wt[0, 0] * eo[0, 1] + wt[0, 1] * eo[0, 3])[None])


@pytest.mark.gpu
@pytest.mark.parametrize("dk,dv", [(128, 64), (64, 128), (128, 8)])
def test_gated_delta_cuda_kernel_matches_reference(dk, dv):
    """The sm_100a recurrence kernel against the PyTorch restatement, including a state carried
    across two calls."""
    from air_rs import ops
    g = torch.Generator().manual_seed(dk + dv)
    BH, L = 3, 37
    q = torch.randn(BH, L, dk, generator=g)
    k = torch.nn.functional.normalize(torch.randn(BH, L, dk, generator=g), dim=-1)
    v = torch.randn(BH, L, dv, generator=g)
    a = torch.rand(BH, L, generator=g) * 0.5 + 0.5
    b = torch.rand(BH, L, generator=g)
    dev = "cuda"
    out, st = ops.gated_delta(q.to(dev), k.to(dev), v.to(dev), a.to(dev), b.to(dev))
    o1, s1 = ops.gated_delta(q[:, :20].to(dev), k[:, :20].to(dev), v[:, :20].to(dev), a[:, :20].to(dev), b[:, :20].to(dev))
    o2, s2 = ops.gated_delta(q[:, 20:].to(dev), k[:, 20:].to(dev), v[:, 20:].to(dev), a[:, 20:].to(dev), b[:, 20:].to(dev), s1)
    for h in range(BH):
        ro, rs = ssm.gated_delta_rule_ref(q[h], k[h], v[h], a[h], b[h])
        torch.testing.assert_close(out[h].cpu(), ro, rtol=1e-4, atol=1e-4)
        torch.testing.assert_close(st[h].cpu(), rs, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(torch.cat([o1, o2], 1), out, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(s2, st, rtol=1e-5, atol=1e-5)
