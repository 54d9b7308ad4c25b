"""GGUF container and quant block codecs (CPU)."""
import struct

import pytest
import torch

from air_rs.gguf import GGMLType, GGUFWriter, read_gguf, quantize, dequantize, tensor_nbytes
from air_rs.gguf.quants import pack_k4_scales, unpack_k4_scales
from air_rs.models.config import ModelConfig, tiny_llama
from air_rs.models.random_init import write_random_gguf


def test_k4_scale_pack_roundtrip():
    g = torch.Generator().manual_seed(0)
    sc = torch.randint(0, 64, (100, 8), generator=g)
    mn = torch.randint(0, 64, (100, 8), generator=g)
    s2, m2 = unpack_k4_scales(pack_k4_scales(sc, mn))
    assert torch.equal(s2, sc.int()) and torch.equal(m2, mn.int())


@pytest.mark.parametrize("qt,tol", [(GGMLType.Q8_0, 0.02), (GGMLType.Q4_K, 0.12), (GGMLType.Q6_K, 0.04),
                                    (GGMLType.F16, 1e-3), (GGMLType.BF16, 1e-2)])
def test_quant_roundtrip(qt, tol):
    x = torch.randn(16, 512) * 0.02
    raw = quantize(x, qt)
    assert raw.shape[-1] == tensor_nbytes(qt, 512)
    y = dequantize(raw, qt)
    rel = (y - x).norm() / x.norm()
    assert rel < tol


def test_q4k_layout_by_hand():
    # one block: d=1, dmin=0.5, sub-block j has scale j+1 and min j; nibble q = element index % 16
    d = torch.tensor([1.0], dtype=torch.float16).view(torch.uint8)
    dmin = torch.tensor([0.5], dtype=torch.float16).view(torch.uint8)
    sc = torch.arange(1, 9).view(1, 8)
    mn = torch.arange(0, 8).view(1, 8)
    packed = pack_k4_scales(sc, mn).view(-1)
    q = torch.arange(256) % 16
    qs = torch.zeros(128, dtype=torch.uint8)
    for j in range(4):
        lo = q[64 * j: 64 * j + 32]
        hi = q[64 * j + 32: 64 * j + 64]
        qs[32 * j: 32 * j + 32] = (lo | (hi << 4)).to(torch.uint8)
    raw = torch.cat([d, dmin, packed, qs]).view(1, 144)
    y = dequantize(raw, GGMLType.Q4_K)[0]
    sub = torch.arange(256) // 32
    ref = (sub + 1).float() * q.float() - 0.5 * sub.float()
    assert torch.allclose(y, ref)


def test_legacy_dequant_shapes():
    for qt in (GGMLType.Q4_0, GGMLType.Q4_1, GGMLType.Q5_0, GGMLType.Q5_1, GGMLType.Q2_K,
               GGMLType.Q3_K, GGMLType.Q5_K, GGMLType.Q8_K):
        nb = tensor_nbytes(qt, 512)
        raw = torch.randint(0, 255, (3, nb), dtype=torch.uint8)
        # make the f16 scales finite
        y = dequantize(raw, qt)
        assert y.shape == (3, 512)


def test_writer_reader_roundtrip(tmp_path):
    p = tmp_path / "m.gguf"
    w = GGUFWriter(str(p), arch="llama")
    w.add("llama.block_count", 3)
    w.add("llama.rope.freq_base", 10000.0)
    w.add("tokenizer.ggml.tokens", ["a", "b", "c"])
    w.add("some.ints", [1, 2, 3])
    x = torch.randn(4, 64)
    w.add_tensor("t.weight", quantize(x, GGMLType.Q8_0), (4, 64), GGMLType.Q8_0)
    w.add_tensor("n.weight", x[0].contiguous().view(torch.uint8), (64,), GGMLType.F32)
    w.write()
    g = read_gguf(str(p))
    assert g.metadata["llama.block_count"] == 3
    assert g.metadata["tokenizer.ggml.tokens"] == ["a", "b", "c"]
    assert g.metadata["some.ints"] == [1, 2, 3]
    assert g.tensors["t.weight"].shape == (64, 4)
    assert g.tensors["t.weight"].offset % 32 == 0
    torch.testing.assert_close(g.dequantize("n.weight"), x[0])
    torch.testing.assert_close(g.dequantize("t.weight"), dequantize(quantize(x, GGMLType.Q8_0), GGMLType.Q8_0))


def test_config_from_metadata_defaults():
    cfg = ModelConfig.from_gguf_metadata({"general.architecture": "llama"})
    assert (cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.hidden_dim) == (32, 32, 32, 4096)
    assert cfg.rope_theta == 500000.0 and cfg.eos_token_id == 2 and cfg.intermediate_dim == 11008
    cfg = ModelConfig.from_gguf_metadata({"general.architecture": "qwen2"})
    assert cfg.rope_theta == 1000000.0
    cfg = ModelConfig.from_gguf_metadata({"general.architecture": "llama", "llama.expert_count": 8,
                                          "llama.expert_used_count": 2})
    assert cfg.ffn_type.value == "softmax_moe" and cfg.moe_top_k == 2


def test_random_gguf_file(tmp_path):
    cfg = tiny_llama()
    p = write_random_gguf(str(tmp_path / "tiny.gguf"), cfg, GGMLType.Q8_0, seed=0)
    g = read_gguf(p)
    c2 = ModelConfig.from_gguf_metadata(g.metadata)
    assert (c2.n_layers, c2.hidden_dim, c2.n_heads, c2.n_kv_heads, c2.head_dim, c2.intermediate_dim,
            c2.vocab_size, c2.rope_theta) == (2, 256, 4, 2, 64, 688, 4096, 10000.0)
    assert g.tensors["blk.0.attn_q.weight"].qtype == GGMLType.Q8_0
    assert torch.equal(g.dequantize("blk.1.ffn_norm.weight"), torch.ones(256))
