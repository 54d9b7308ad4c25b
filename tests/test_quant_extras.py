"""Extra quantisation codecs (reference tests in src/fp8.rs, src/w8a8.rs, src/ternary.rs,
src/turbo_quant.rs, src/hqq.rs, src/aqlm.rs, src/alt_quant.rs, src/iso_quant.rs)."""
import math

import pytest
import torch

from air_rs.gguf import GGMLType, dequantize
from air_rs.quant import (Fp8Linear, TernaryMatMul, e4m3_from_f32, e4m3_to_f32, e5m2_from_f32, e5m2_to_f32,
                          kv_q8_0_decode, kv_q8_0_encode, pack_trits, quantize_f32_to_i8, unpack_trits, w8a8_matmul)
from air_rs.quant import codecs as C


def test_fp8_matches_torch_dtypes():
    g = torch.Generator().manual_seed(0)
    x = torch.cat([torch.randn(4000, generator=g) * s for s in (1e-3, 0.1, 3.0, 100.0)])
    x = torch.cat([x, torch.tensor([0.0, -0.0, 448.0, -448.0, 2.0 ** -9, 1.0625, 1.1875])])
    b = e4m3_from_f32(x)
    ref = x.to(torch.float8_e4m3fn).view(torch.uint8)
    assert torch.equal(b, ref)
    torch.testing.assert_close(e4m3_to_f32(b), x.to(torch.float8_e4m3fn).float())
    y = x.clamp(-57344, 57344)
    assert torch.equal(e5m2_from_f32(y), y.to(torch.float8_e5m2).view(torch.uint8))
    assert float(e4m3_to_f32(e4m3_from_f32(torch.tensor(1e6)))) == 448.0     # saturates
    assert math.isnan(float(e4m3_to_f32(torch.tensor(0x7F, dtype=torch.uint8))))
    w = torch.randn(16, 32, generator=g)
    lin = Fp8Linear(w)
    assert float((lin.dequantize() - w).abs().max()) < 0.07 * float(w.abs().max())


def test_w8a8_and_kv_q8():
    g = torch.Generator().manual_seed(1)
    x, w = torch.randn(5, 64, generator=g), torch.randn(64, 7, generator=g)
    xq, sx = quantize_f32_to_i8(x)
    wq, sw = quantize_f32_to_i8(w)
    out = w8a8_matmul(xq, wq, sx, sw)
    assert float((out - x @ w).abs().max()) < 0.05 * float((x @ w).abs().max())
    assert quantize_f32_to_i8(torch.zeros(3))[1] == 1.0
    kv = torch.randn(2, 4, 64, generator=g)
    q, s = kv_q8_0_encode(kv)
    assert q.dtype == torch.int8 and s.shape == (2, 4, 2)
    assert float((kv_q8_0_decode(q, s) - kv).abs().max()) <= float(s.max()) * 0.5 + 1e-6


def test_ternary_pack_and_matmul():
    t = torch.tensor([-1, 0, 1, 1, -1, 0, 0, 1], dtype=torch.int8)
    p = pack_trits(t)
    assert p.tolist()[0] == 0 * 1 + 1 * 3 + 2 * 9 + 2 * 27 + 0 * 81 and p.numel() == 2
    assert torch.equal(unpack_trits(p, 8), t)
    g = torch.Generator().manual_seed(2)
    w = torch.randn(6, 20, generator=g)
    mm = TernaryMatMul.from_float(w)
    xq = torch.randint(-127, 128, (3, 20), generator=g, dtype=torch.int8)
    ref = xq.float() @ (mm.trits.float() * mm.scales[:, None]).t()
    torch.testing.assert_close(mm.matmul_i8(xq, 1.0), ref)


def test_turboquant_roundtrip():
    x = torch.randn(100, generator=torch.Generator().manual_seed(3))
    blocks = C.tq4_compress(x)
    assert len(blocks) == 4 and blocks[0][1].numel() == 16
    y = C.tq4_decompress(blocks, 100)
    assert float(((y - x) ** 2).mean()) < 0.02 * float((x ** 2).mean()) + 1e-4
    c = C.lloyd_max(torch.randn(5000, generator=torch.Generator().manual_seed(4)), levels=4)
    # the 4-level Lloyd-Max quantiser of N(0,1) has centroids near +-0.453, +-1.510
    assert abs(abs(float(c[0])) - 1.510) < 0.1 and abs(abs(float(c[1])) - 0.453) < 0.06


def test_hqq_pack_unpack_and_dequant():
    for nb in (1, 2, 3, 4, 8):
        codes = torch.randint(0, 2 ** nb, (37,), generator=torch.Generator().manual_seed(nb)).to(torch.uint8)
        assert torch.equal(C.unpack_bits(C.pack_bits(codes, nb), nb, 37), codes)
    w = torch.randn(8, 100, generator=torch.Generator().manual_seed(5))
    packed, scale, zero = C.hqq_quantize(w, 4, 32)
    d = C.hqq_dequantize(packed, 4, scale, zero, (8, 100), 32, axis=0)
    assert float((d - w).abs().max()) <= float(scale.max()) * 0.51


def test_aqlm_additive_quantisation():
    w = torch.randn(32, 64, generator=torch.Generator().manual_seed(6))
    codes, books, scales = C.aqlm_quantize(w, n_codebooks=2)
    d = C.aqlm_dequantize(codes, books, scales)
    assert codes.shape == (32, 8, 2) and books.shape == (2, 256, 8)
    rel = float((d - w).norm() / w.norm())
    one = C.aqlm_dequantize(codes[..., :1], books[:1], scales)
    assert rel < float((one - w).norm() / w.norm()) < 1.0        # the second codebook helps


def test_gptq_and_awq_layouts():
    g = torch.Generator().manual_seed(7)
    K, N, gs = 32, 16, 16
    q = torch.randint(0, 16, (K, N), generator=g)
    z = torch.randint(1, 16, (K // gs, N), generator=g)       # GPTQ stores z-1 in 4 bits
    s = torch.rand(K // gs, N, generator=g) + 0.5
    ref = ((q - z[torch.arange(K) // gs]) * s[torch.arange(K) // gs]).t()
    qweight = C.pack_int32(q.reshape(K // 8, 8, N).permute(0, 2, 1))             # packed along K
    qzeros = C.pack_int32((z - 1).reshape(K // gs, N // 8, 8))                    # along N, minus one
    torch.testing.assert_close(C.gptq_dequantize(qweight, qzeros, s, group_size=gs), ref.float())
    order = torch.tensor(C.AWQ_ORDER)
    aw = C.pack_int32(q.reshape(K, N // 8, 8)[..., order])
    az = C.pack_int32(z.reshape(K // gs, N // 8, 8)[..., order])
    torch.testing.assert_close(C.awq_dequantize(aw, az, s, group_size=gs), ref.float())


def test_isoquant_preserves_dot_products():
    iq = C.IsoQuant(64, seed=1)
    assert torch.allclose(iq.R @ iq.R.t(), torch.eye(64), atol=1e-5)
    a, b = torch.randn(2, 64, generator=torch.Generator().manual_seed(8))
    assert abs(float(iq.project(a) @ iq.project(b)) - float(a @ b)) < 1e-3
    q, s = iq.encode(a[None])
    assert float((iq.reconstruct(q, s)[0] - a).abs().max()) < 0.05


def test_iq4_formats_against_definition():
    g = torch.Generator().manual_seed(9)
    raw = torch.randint(0, 256, (2, 18), generator=g, dtype=torch.uint8)
    raw[:, 0:2] = torch.tensor([0x00, 0x3C], dtype=torch.uint8)                  # d = 1.0
    out = dequantize(raw, GGMLType.IQ4_NL).reshape(2, 32)
    from air_rs.gguf.quants import IQ4_NL_VALUES
    assert float(out[0, 0]) == float(IQ4_NL_VALUES[int(raw[0, 2]) & 0xF])
    assert float(out[0, 16]) == float(IQ4_NL_VALUES[int(raw[0, 2]) >> 4])
    raw = torch.randint(0, 256, (1, 136), generator=g, dtype=torch.uint8)
    raw[:, 0:2] = torch.tensor([0x00, 0x3C], dtype=torch.uint8)
    out = dequantize(raw, GGMLType.IQ4_XS).reshape(256)
    sh = int(raw[0, 2]) | (int(raw[0, 3]) << 8)
    ls = (int(raw[0, 4]) & 0xF) | ((sh & 3) << 4)
    assert float(out[0]) == (ls - 32) * float(IQ4_NL_VALUES[int(raw[0, 8]) & 0xF])


def test_fp8_b128_block_format():
    """Block-scaled FP8 (internal type FP8_E4M3_B128: f32 multiplier + 128 E4M3 codes per
    block): round trip within E4M3's relative step, and a 128 x 128-tile fp8 checkpoint maps
    onto it with its codes unchanged (exact)."""
    import torch
    from air_rs.gguf import GGMLType, dequantize, quantize
    from air_rs.gguf.quants import fp8_b128_from_tiles
    from air_rs.quant.fp8 import block_dequantize_fp8, block_quantize_fp8
    g = torch.Generator().manual_seed(0)
    x = torch.randn(6, 384, generator=g)
    raw = quantize(x, GGMLType.FP8_E4M3_B128)
    assert raw.shape == (6, 3 * 132)
    y = dequantize(raw, GGMLType.FP8_E4M3_B128)
    blk = x.reshape(6, 3, 128).abs().amax(-1, keepdim=True)
    assert float(((y - x).reshape(6, 3, 128).abs() / blk).max()) <= 1 / 14 + 1e-6   # half an E4M3 step at 448
    w = torch.randn(256, 384, generator=g)
    codes, s_inv = block_quantize_fp8(w)
    r2 = fp8_b128_from_tiles(codes, s_inv)
    torch.testing.assert_close(dequantize(r2, GGMLType.FP8_E4M3_B128), block_dequantize_fp8(codes, s_inv))
