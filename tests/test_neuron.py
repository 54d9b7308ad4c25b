"""Neuron-predicate loading (reference src/neuron_predicate.rs tests)."""
import torch

from air_rs.stream.neuron import (BUNDLE_SIZE, BundleMap, NeuronMask, NeuronPredictor, PredicateCache,
                                  sparse_ffn)


def test_mask_bundle_rounding():
    s = torch.zeros(300)
    s[5] = 0.9
    s[130] = 0.7
    m = NeuronMask.from_scores(s, 0.5)
    assert m.n_bundles() == 5 and m.active_bundles() == 2 and m.active_count() == 128
    assert m.is_active(0) and m.is_active(63) and not m.is_active(64) and m.is_active(191)
    assert abs(m.sparsity() - (1 - 128 / 300)) < 1e-9
    assert NeuronMask.all_active(300).active_count() == 300 and NeuronMask.all_inactive(10).active_count() == 0
    fb = NeuronMask.from_bundles([True, False, True], 150)
    assert fb.active_count() == 64 + 22


def test_bundle_map_coalesces():
    m = NeuronMask.from_bundles([True, True, False, True, False, True, True, True], 8 * BUNDLE_SIZE)
    bm = BundleMap(m)
    assert bm.n_reads() == 3 and bm.total_bundles == 6
    assert bm.io_ranges(10) == [(0, 1280), (3 * 640, 640), (5 * 640, 1920)]
    assert bm.total_bytes(2) == 6 * 64 * 2


def test_predictor_cache_and_sparse_ffn():
    H, D = 32, 256
    p = NeuronPredictor.random(H, D, seed=1, threshold=0.5)
    h = torch.randn(3, H)
    assert p.scores(h).shape == (3, D)
    m = p.predict(h)
    assert 0 <= m.active_bundles() <= 4
    c = PredicateCache(0.99)
    c.get(0, h[0], p)
    c.get(0, h[0] * 1.001, p)
    c.get(0, -h[0], p)
    assert c.hits == 1 and c.misses == 2
    g = torch.Generator().manual_seed(0)
    wg, wu, wd = torch.randn(D, H, generator=g), torch.randn(D, H, generator=g), torch.randn(H, D, generator=g)
    x = torch.randn(2, H, generator=g)
    dense = (torch.nn.functional.silu(x @ wg.t()) * (x @ wu.t())) @ wd.t()
    torch.testing.assert_close(sparse_ffn(x, wg, wu, wd, NeuronMask.all_active(D)), dense, rtol=1e-4, atol=1e-3)
    half = NeuronMask.from_bundles([True, True, False, False], D)
    act = torch.nn.functional.silu(x @ wg.t()) * (x @ wu.t())
    act[:, 128:] = 0
    torch.testing.assert_close(sparse_ffn(x, wg, wu, wd, half), act @ wd.t(), rtol=1e-4, atol=1e-3)
