"""EXL2-style mixed-width groups, Q4_0 ARM tile orders, PrismML Q1_0 / Q2_0 (reference
src/alt_quant.rs, src/q4_tiled.rs, src/prism_dequant.rs tests)."""
import pytest
import torch

from air_rs.gguf import GGMLType, dequantize, quantize
from air_rs.quant import codecs as C


def test_detect_format():
    assert C.detect_alt_format(["model.q_groups", "x"]) == "exl2"
    assert C.detect_alt_format(["a.qweight", "a.qzeros", "a.scales"]) == "gptq"
    assert C.detect_alt_format(["a.zeros", "a.scales"]) == "awq"
    assert C.detect_alt_format(["a.weight"]) is None


def test_exl2_roundtrip_with_perm():
    g = torch.Generator().manual_seed(0)
    bits = [4, 3, 6, 2]
    K, N = 128, 5
    q = torch.cat([torch.randint(0, 1 << b, (32, N), generator=g) for b in bits])
    scale = torch.rand(4, N, generator=g) * 255
    perm = torch.randperm(K, generator=g)
    groups = torch.tensor([[b, 0] for b in bits])
    w = C.exl2_dequantize(C.exl2_pack(q, bits), scale, 2.0, groups, perm)
    ref = torch.cat([(q[i * 32:(i + 1) * 32].float() - (1 << (b - 1))) * scale[i] * (2.0 / 256)
                     for i, b in enumerate(bits)])
    res = torch.empty_like(ref)
    res[perm] = ref
    torch.testing.assert_close(w, res)


def test_q4_0_tile_orders():
    g = torch.Generator().manual_seed(1)
    nb = 8
    blocks = torch.randint(0, 256, (nb, 18), generator=g, dtype=torch.int64).to(torch.uint8)
    blocks[:, :2] = (torch.rand(nb, generator=g) * 0.1 + 0.01).to(torch.float16).view(torch.uint8).reshape(nb, 2)
    raw = blocks.reshape(-1)
    # row-major (untiled) order: byte i holds codes 2i (low nibble) and 2i + 1 (high nibble)
    d = blocks[:, :2].contiguous().view(torch.float16).float()
    nib = blocks[:, 2:].long()
    codes = torch.stack([nib & 0xF, nib >> 4], -1).reshape(nb, 32)
    ref = ((codes - 8).float() * d).reshape(-1)
    for kind in ("4x4", "4x8", "8x8"):
        torch.testing.assert_close(C.q4_0_tiled_dequantize(C.q4_0_tile(raw, kind), kind), ref)
    # the 4x4 order really moves codes
    assert not torch.equal(C.q4_0_tiled_dequantize(raw, "4x4"), ref)
    with pytest.raises(ValueError):
        C.q4_0_tiled_dequantize(raw, "2x2")


def test_prism_q1_q2():
    blk = torch.zeros(18, dtype=torch.uint8)
    blk[:2] = torch.tensor([1.5], dtype=torch.float16).view(torch.uint8)
    blk[2:] = 0xFF
    assert torch.equal(C.prism_q1_0_dequantize(blk), torch.full((128,), 1.5))
    blk[2] = 0b00000001
    out = C.prism_q1_0_dequantize(blk)
    assert out[0] == 1.5 and out[1] == -1.5
    b2 = torch.zeros(34, dtype=torch.uint8)
    b2[:2] = torch.tensor([2.0], dtype=torch.float16).view(torch.uint8)
    b2[2] = 0b11100100            # codes 0, 1, 2, 3
    o2 = C.prism_q2_0_dequantize(b2)
    assert o2[:4].tolist() == [-2.0, 0.0, 2.0, 4.0] and o2[4] == -2.0
    with pytest.raises(ValueError):
        C.prism_q2_0_dequantize(torch.zeros(33, dtype=torch.uint8))
