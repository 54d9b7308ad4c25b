"""KV warm-tier codecs (reference src/kv_compress.rs tests)."""
import math

import torch

from air_rs.kv.compress import (CompressedKeys, CompressedValues, KvBudgetCalc, QjlKeys, TriageWeights,
                                qjl_projection_matrix, rank_entries, triage_score)


def test_sign_keys_roundtrip_properties():
    g = torch.Generator().manual_seed(0)
    k = torch.randn(50, 128, generator=g)
    c = CompressedKeys.compress(k)
    r = c.decompress()
    assert r.shape == k.shape
    # signs about the mean are kept, mean preserved per row
    assert bool(((k >= k.mean(-1, keepdim=True)) == (r >= c.mean[:, None])).all())
    torch.testing.assert_close(r.mean(-1), k.mean(-1), atol=0.2, rtol=0)
    cos = torch.nn.functional.cosine_similarity(r - c.mean[:, None], k - k.mean(-1, keepdim=True))
    assert float(cos.mean()) > 0.7
    assert c.compression_ratio() > 10


def test_values_8bit_error_bound():
    v = torch.randn(40, 64) * 3
    c = CompressedValues.compress(v)
    err = (c.decompress() - v).abs().max(-1).values
    assert bool((err <= c.scale / 2 + 1e-5).all())
    const = CompressedValues.compress(torch.full((2, 8), 1.25))
    assert torch.allclose(const.decompress(), torch.full((2, 8), 1.25))
    assert abs(c.compression_ratio() - 2 * 64 / (64 + 8)) < 1e-9


def test_qjl_similarity_estimate():
    g = torch.Generator().manual_seed(3)
    d, m = 128, 1024
    R = qjl_projection_matrix(m, d, seed=1)
    q = torch.randn(d, generator=g)
    k = torch.stack([q, -q, torch.randn(d, generator=g), 0.5 * q + 0.1 * torch.randn(d, generator=g)])
    c = QjlKeys.compress(k, R)
    est = c.approx_cos_sim(QjlKeys.query_bits(q[None], R)[0])
    true = torch.nn.functional.cosine_similarity(k, q[None])
    assert float((est - true).abs().max()) < 0.15
    assert est[0] > 0.99 and est[1] < -0.99
    dots = c.approx_dot(QjlKeys.query_bits(q[None], R)[0], float(q.norm()))
    assert int(dots.argmax()) == int((k @ q).argmax())
    assert c.size_bytes() == 4 * (m // 8) + 16


def test_triage_and_budget():
    w = TriageWeights()
    s = float(triage_score(w, 0.5, 10, 10, 3))
    assert abs(s - (0.25 + 0.30 + 0.20)) < 1e-9
    ranked = rank_entries(w, [(100, 0.1, 0), (5, 0.1, 0), (200, 0.9, 10)], 10)
    assert [p for p, _ in ranked] == [200, 5, 100]
    b = KvBudgetCalc(80, 8, 128)
    assert b.bytes_per_token() == 80 * 2 * 8 * 128 * 2
    assert abs(b.total_mb(4096) - 4096 * 327680 / 2**20) < 1e-6
    assert b.compressed_warm_mb(4096) < b.total_mb(4096) / 1.8
    assert b.fits(4096, 2000) and not b.fits(32768, 2000) and b.fits(8192, 2000, compressed=True)
