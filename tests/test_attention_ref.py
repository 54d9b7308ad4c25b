"""Split-K flash decoding and blockwise attention oracles (reference src/flash_decode.rs,
src/chunked_attn.rs tests) against dense attention."""
import pytest
import torch

from air_rs.models.attention_ref import (ChunkedAttentionConfig, blockwise_attention, flash_decode,
                                         max_abs_error, memory_reduction_factor, peak_memory_bytes,
                                         reference_attention)
from air_rs.models.reference import attention_reference


@pytest.mark.parametrize("T,chunk", [(1, 64), (63, 64), (64, 64), (1000, 64), (300, 7)])
def test_flash_decode_matches_dense(T, chunk):
    g = torch.Generator().manual_seed(T)
    q = torch.randn(8, 64, generator=g)
    k = torch.randn(T, 2, 64, generator=g)
    v = torch.randn(T, 2, 64, generator=g)
    assert max_abs_error(flash_decode(q, k, v, chunk), reference_attention(q, k, v)) < 1e-4


@pytest.mark.parametrize("Sq,Skv,block,causal", [(1, 1000, 512, True), (37, 37, 16, True), (20, 70, 8, True),
                                                 (5, 33, 512, False)])
def test_blockwise_matches_dense(Sq, Skv, block, causal):
    g = torch.Generator().manual_seed(Sq + Skv)
    cfg = ChunkedAttentionConfig(block_size=block, n_heads=8, n_kv_heads=2, head_dim=32, causal=causal)
    q = torch.randn(Sq, 8, 32, generator=g)
    k = torch.randn(Skv, 2, 32, generator=g)
    v = torch.randn(Skv, 2, 32, generator=g)
    ref = attention_reference(q, k, v, causal=causal)
    torch.testing.assert_close(blockwise_attention(q, k, v, cfg), ref, rtol=1e-4, atol=1e-5)


def test_config_and_memory():
    cfg = ChunkedAttentionConfig()
    assert cfg.gqa_groups() == 4 and abs(cfg.scale() - 128 ** -0.5) < 1e-9
    assert peak_memory_bytes(1, 8192, cfg) == 512 * 32 * 4
    assert memory_reduction_factor(1, 8192, cfg) == 16.0 and memory_reduction_factor(1, 100, cfg) == 1.0
    for bad in (dict(block_size=0), dict(head_dim=0), dict(n_heads=6, n_kv_heads=4)):
        with pytest.raises(ValueError):
            ChunkedAttentionConfig(**bad).validate()
