"""GGUF quant block codecs, vectorised over whole tensors with torch.

The block layouts are the GGUF/ggml ones (they are the checkpoint format, so they
cannot differ): the reference reads them through candle's ``k_quants`` in
``src/weight_streamer.rs:504-600``. Every function takes/returns torch tensors and
therefore runs on the CPU or, for the random-init benchmark weights, on the GPU.

``raw`` tensors are ``uint8`` with the last dimension holding whole blocks of one row.
Dequantisers return ``float32`` with the last dimension = row length.

Quantisers in this file are simple, deterministic round-to-nearest schemes of our own
(min/max per sub-block for the K-quants); they emit format-valid blocks that any GGUF
reader decodes, but they are not llama.cpp's iterative search quantisers.
"""
from __future__ import annotations

import torch

from .constants import GGMLType, QK_K, BLOCK_GEOMETRY


def _blocks(raw: torch.Tensor, nbytes: int) -> torch.Tensor:
    if raw.dtype != torch.uint8:
        raise TypeError("raw block tensor must be uint8")
    if raw.shape[-1] % nbytes:
        raise ValueError(f"row of {raw.shape[-1]} bytes is not a multiple of the block size {nbytes}")
    return raw.reshape(*raw.shape[:-1], raw.shape[-1] // nbytes, nbytes)


def _f16(b: torch.Tensor) -> torch.Tensor:
    """Two uint8 columns (little endian) -> float32."""
    return b.contiguous().view(torch.float16).squeeze(-1).float()


def _f32(b: torch.Tensor) -> torch.Tensor:
    return b.contiguous().view(torch.float32).squeeze(-1)


def _u32(b: torch.Tensor) -> torch.Tensor:
    b = b.to(torch.int64)
    return b[..., 0] | (b[..., 1] << 8) | (b[..., 2] << 16) | (b[..., 3] << 24)


def _flat(y: torch.Tensor) -> torch.Tensor:
    return y.reshape(*y.shape[:-2], -1)


# ---------------------------------------------------------------------------
# legacy 32-element blocks
# ---------------------------------------------------------------------------

def dequantize_q8_0(raw: torch.Tensor) -> torch.Tensor:
    b = _blocks(raw, 34)
    d = _f16(b[..., 0:2])
    q = b[..., 2:34].contiguous().view(torch.int8).float()
    return _flat(q * d.unsqueeze(-1))


def quantize_q8_0(x: torch.Tensor) -> torch.Tensor:
    """Round-to-nearest Q8_0: d = absmax/127 per 32 elements."""
    x = x.float()
    xb = x.reshape(*x.shape[:-1], x.shape[-1] // 32, 32)
    amax = xb.abs().amax(-1)
    d = amax / 127.0
    inv = torch.where(d > 0, 1.0 / d, torch.zeros_like(d))
    q = torch.round(xb * inv.unsqueeze(-1)).clamp(-127, 127).to(torch.int8)
    dh = d.to(torch.float16).unsqueeze(-1).view(torch.uint8)
    out = torch.cat([dh, q.view(torch.uint8)], -1)
    return out.reshape(*x.shape[:-1], -1)


def dequantize_q4_0(raw: torch.Tensor) -> torch.Tensor:
    b = _blocks(raw, 18)
    d = _f16(b[..., 0:2]).unsqueeze(-1)
    qs = b[..., 2:18].to(torch.int16)
    lo = (qs & 0xF) - 8
    hi = (qs >> 4) - 8
    return _flat(torch.cat([lo, hi], -1).float() * d)


def dequantize_q4_1(raw: torch.Tensor) -> torch.Tensor:
    b = _blocks(raw, 20)
    d = _f16(b[..., 0:2]).unsqueeze(-1)
    m = _f16(b[..., 2:4]).unsqueeze(-1)
    qs = b[..., 4:20].to(torch.int16)
    q = torch.cat([qs & 0xF, qs >> 4], -1).float()
    return _flat(q * d + m)


def _q5_high_bits(qh: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    j = torch.arange(16, device=qh.device)
    h = qh.unsqueeze(-1)
    h0 = ((h >> j) << 4) & 0x10
    h1 = (h >> (j + 12)) & 0x10
    return h0, h1


def dequantize_q5_0(raw: torch.Tensor) -> torch.Tensor:
    b = _blocks(raw, 22)
    d = _f16(b[..., 0:2]).unsqueeze(-1)
    h0, h1 = _q5_high_bits(_u32(b[..., 2:6]))
    qs = b[..., 6:22].to(torch.int64)
    lo = ((qs & 0xF) | h0) - 16
    hi = ((qs >> 4) | h1) - 16
    return _flat(torch.cat([lo, hi], -1).float() * d)


def dequantize_q5_1(raw: torch.Tensor) -> torch.Tensor:
    b = _blocks(raw, 24)
    d = _f16(b[..., 0:2]).unsqueeze(-1)
    m = _f16(b[..., 2:4]).unsqueeze(-1)
    h0, h1 = _q5_high_bits(_u32(b[..., 4:8]))
    qs = b[..., 8:24].to(torch.int64)
    q = torch.cat([(qs & 0xF) | h0, (qs >> 4) | h1], -1).float()
    return _flat(q * d + m)


# ---------------------------------------------------------------------------
# K-quants (256-element super-blocks)
# ---------------------------------------------------------------------------

def unpack_k4_scales(sc12: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """12 packed bytes -> 8 six-bit scales and 8 six-bit mins (Q4_K / Q5_K)."""
    q = sc12.to(torch.int32)
    sc_lo = q[..., 0:4] & 63
    m_lo = q[..., 4:8] & 63
    sc_hi = (q[..., 8:12] & 0xF) | ((q[..., 0:4] >> 6) << 4)
    m_hi = (q[..., 8:12] >> 4) | ((q[..., 4:8] >> 6) << 4)
    return torch.cat([sc_lo, sc_hi], -1), torch.cat([m_lo, m_hi], -1)


def pack_k4_scales(sc: torch.Tensor, mn: torch.Tensor) -> torch.Tensor:
    """Inverse of :func:`unpack_k4_scales` (inputs int in [0, 63])."""
    sc = sc.to(torch.int32)
    mn = mn.to(torch.int32)
    b0_3 = (sc[..., 0:4] & 63) | ((sc[..., 4:8] >> 4) << 6)
    b4_7 = (mn[..., 0:4] & 63) | ((mn[..., 4:8] >> 4) << 6)
    b8_11 = (sc[..., 4:8] & 0xF) | ((mn[..., 4:8] & 0xF) << 4)
    return torch.cat([b0_3, b4_7, b8_11], -1).to(torch.uint8)


def dequantize_q4_k(raw: torch.Tensor) -> torch.Tensor:
    b = _blocks(raw, 144)
    d = _f16(b[..., 0:2]).unsqueeze(-1)
    dmin = _f16(b[..., 2:4]).unsqueeze(-1)
    sc, mn = unpack_k4_scales(b[..., 4:16])
    qs = b[..., 16:144].reshape(*b.shape[:-1], 4, 32).to(torch.int16)
    q = torch.stack([qs & 0xF, qs >> 4], -2).reshape(*b.shape[:-1], 8, 32).float()
    y = q * (d * sc.float()).unsqueeze(-1) - (dmin * mn.float()).unsqueeze(-1)
    return _flat(y.reshape(*b.shape[:-1], 256))


def quantize_q4_k(x: torch.Tensor) -> torch.Tensor:
    """Min/max Q4_K: per 32-sub-block affine 4-bit codes, 6-bit scales/mins per super-block."""
    x = x.float()
    shp = x.shape[:-1]
    nb = x.shape[-1] // QK_K
    xb = x.reshape(*shp, nb, 8, 32)
    lo = xb.amin(-1).clamp(max=0.0)
    hi = xb.amax(-1)
    scale = (hi - lo) / 15.0
    mins = -lo
    d = scale.amax(-1) / 63.0
    dmin = mins.amax(-1) / 63.0
    d16 = d.to(torch.float16)
    dmin16 = dmin.to(torch.float16)
    df = d16.float().unsqueeze(-1)
    dmf = dmin16.float().unsqueeze(-1)
    sc = torch.where(df > 0, torch.round(scale / df.clamp_min(1e-30)), torch.zeros_like(scale)).clamp(0, 63)
    mq = torch.where(dmf > 0, torch.round(mins / dmf.clamp_min(1e-30)), torch.zeros_like(mins)).clamp(0, 63)
    eff_s = (df * sc).unsqueeze(-1)
    eff_m = (dmf * mq).unsqueeze(-1)
    q = torch.where(eff_s > 0, torch.round((xb + eff_m) / eff_s.clamp_min(1e-30)), torch.zeros_like(xb))
    q = q.clamp(0, 15).to(torch.uint8).reshape(*shp, nb, 4, 2, 32)
    qs = (q[..., 0, :] | (q[..., 1, :] << 4)).reshape(*shp, nb, 128)
    head = torch.cat([
        d16.unsqueeze(-1).view(torch.uint8),
        dmin16.unsqueeze(-1).view(torch.uint8),
        pack_k4_scales(sc, mq),
    ], -1)
    return torch.cat([head, qs], -1).reshape(*shp, nb * 144)


def dequantize_q5_k(raw: torch.Tensor) -> torch.Tensor:
    b = _blocks(raw, 176)
    d = _f16(b[..., 0:2]).unsqueeze(-1)
    dmin = _f16(b[..., 2:4]).unsqueeze(-1)
    sc, mn = unpack_k4_scales(b[..., 4:16])
    qh = b[..., 16:48].to(torch.int16)  # [.., 32]
    qs = b[..., 48:176].reshape(*b.shape[:-1], 4, 32).to(torch.int16)
    sub = torch.arange(8, device=raw.device)
    hb = ((qh.unsqueeze(-2) >> sub.view(8, 1)) & 1) * 16  # [..,8,32]
    low = torch.stack([qs & 0xF, qs >> 4], -2).reshape(*b.shape[:-1], 8, 32)
    q = (low + hb).float()
    y = q * (d * sc.float()).unsqueeze(-1) - (dmin * mn.float()).unsqueeze(-1)
    return _flat(y.reshape(*b.shape[:-1], 256))


def dequantize_q6_k(raw: torch.Tensor) -> torch.Tensor:
    b = _blocks(raw, 210)
    ql = b[..., 0:128].reshape(*b.shape[:-1], 2, 64).to(torch.int16)
    qh = b[..., 128:192].reshape(*b.shape[:-1], 2, 32).to(torch.int16)
    sc = b[..., 192:208].contiguous().view(torch.int8).float().reshape(*b.shape[:-1], 2, 8)
    d = _f16(b[..., 208:210]).unsqueeze(-1).unsqueeze(-1)
    q1 = (ql[..., 0:32] & 0xF) | (((qh >> 0) & 3) << 4)
    q2 = (ql[..., 32:64] & 0xF) | (((qh >> 2) & 3) << 4)
    q3 = (ql[..., 0:32] >> 4) | (((qh >> 4) & 3) << 4)
    q4 = (ql[..., 32:64] >> 4) | (((qh >> 6) & 3) << 4)
    q = torch.stack([q1, q2, q3, q4], -2).float() - 32.0  # [.., 2, 4, 32]
    # scale index within a half: (l // 16) + 2 * quarter
    s = sc.reshape(*b.shape[:-1], 2, 4, 2).unsqueeze(-1).expand(*b.shape[:-1], 2, 4, 2, 16)
    s = s.reshape(*b.shape[:-1], 2, 4, 32)
    y = d.unsqueeze(-1) * s * q
    return _flat(y.reshape(*b.shape[:-1], 256))


def quantize_q6_k(x: torch.Tensor) -> torch.Tensor:
    """Absmax Q6_K: 16-element sub-blocks with int8 scales, 6-bit symmetric codes."""
    x = x.float()
    shp = x.shape[:-1]
    nb = x.shape[-1] // QK_K
    xb = x.reshape(*shp, nb, 16, 16)
    amax = xb.abs().amax(-1)
    scale = amax / 31.0
    d = scale.amax(-1) / 127.0
    d16 = d.to(torch.float16)
    df = d16.float().unsqueeze(-1)
    sc = torch.where(df > 0, torch.round(scale / df.clamp_min(1e-30)), torch.zeros_like(scale)).clamp(-128, 127)
    eff = (df * sc).unsqueeze(-1)
    q = torch.where(eff != 0, torch.round(xb / torch.where(eff != 0, eff, torch.ones_like(eff))), torch.zeros_like(xb))
    q = (q.clamp(-32, 31) + 32).to(torch.int16).reshape(*shp, nb, 2, 4, 32)  # half, quarter, l
    q1, q2, q3, q4 = q[..., 0, :], q[..., 1, :], q[..., 2, :], q[..., 3, :]
    ql_a = (q1 & 0xF) | ((q3 & 0xF) << 4)
    ql_b = (q2 & 0xF) | ((q4 & 0xF) << 4)
    ql = torch.cat([ql_a, ql_b], -1).reshape(*shp, nb, 128)
    qh = ((q1 >> 4) & 3) | (((q2 >> 4) & 3) << 2) | (((q3 >> 4) & 3) << 4) | (((q4 >> 4) & 3) << 6)
    qh = qh.reshape(*shp, nb, 64)
    out = torch.cat([
        ql.to(torch.uint8), qh.to(torch.uint8),
        sc.to(torch.int8).view(torch.uint8),
        d16.unsqueeze(-1).view(torch.uint8),
    ], -1)
    return out.reshape(*shp, nb * 210)


def dequantize_q2_k(raw: torch.Tensor) -> torch.Tensor:
    b = _blocks(raw, 84)
    scales = b[..., 0:16].to(torch.int16)
    qs = b[..., 16:80].reshape(*b.shape[:-1], 2, 32).to(torch.int16)
    d = _f16(b[..., 80:82])[..., None, None, None]
    dmin = _f16(b[..., 82:84])[..., None, None, None]
    shifts = torch.tensor([0, 2, 4, 6], device=raw.device).view(1, 4, 1)
    q = (qs.unsqueeze(-2) >> shifts) & 3  # [.., 2, 4, 32]
    sc = scales.reshape(*b.shape[:-1], 2, 4, 2)
    dl = (sc & 0xF).float().repeat_interleave(16, -1)
    ml = (sc >> 4).float().repeat_interleave(16, -1)
    y = d * dl * q.float() - dmin * ml
    return _flat(y.reshape(*b.shape[:-1], 256))


def dequantize_q3_k(raw: torch.Tensor) -> torch.Tensor:
    b = _blocks(raw, 110)
    hm = b[..., 0:32].to(torch.int16)
    qs = b[..., 32:96].reshape(*b.shape[:-1], 2, 32).to(torch.int16)
    s = b[..., 96:108].to(torch.int32)
    d = _f16(b[..., 108:110])[..., None, None, None]
    # 16 six-bit scales: low nibbles from bytes 0..7, high 2 bits from bytes 8..11
    low = torch.cat([s[..., 0:8] & 0xF, s[..., 0:8] >> 4], -1)
    hib = s[..., 8:12]
    hi = torch.stack([(hib >> (2 * k)) & 3 for k in range(4)], -2).reshape(*b.shape[:-1], 16)
    scales = (low | (hi << 4)) - 32
    shifts = torch.tensor([0, 2, 4, 6], device=raw.device).view(1, 4, 1)
    q = (qs.unsqueeze(-2) >> shifts) & 3  # [.., 2, 4, 32]
    bit = torch.arange(8, device=raw.device).view(2, 4, 1)
    hset = (hm.reshape(*b.shape[:-1], 1, 1, 32) >> bit) & 1
    q = q - torch.where(hset > 0, 0, 4)
    sc = scales.reshape(*b.shape[:-1], 2, 4, 2).float().repeat_interleave(16, -1)
    y = d * sc * q.float()
    return _flat(y.reshape(*b.shape[:-1], 256))


def dequantize_q8_k(raw: torch.Tensor) -> torch.Tensor:
    b = _blocks(raw, 292)
    d = _f32(b[..., 0:4]).unsqueeze(-1)
    q = b[..., 4:260].contiguous().view(torch.int8).float()
    return _flat(q * d)


# ---------------------------------------------------------------------------
# IQ4 non-linear 4-bit formats: a fixed 16-entry int8 codebook (part of the GGUF format
# definition) scaled per 32-element block (IQ4_NL) or per 32 within a 256 super-block with
# 6-bit scales (IQ4_XS)
# ---------------------------------------------------------------------------

IQ4_NL_VALUES = torch.tensor([-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113],
                             dtype=torch.float32)


def _iq4_nibbles(qs: torch.Tensor) -> torch.Tensor:
    """16 bytes -> 32 codebook values: low nibbles first, then high nibbles."""
    lo, hi = (qs & 0xF).long(), (qs >> 4).long()
    return IQ4_NL_VALUES[torch.cat([lo, hi], -1)]


def dequantize_iq4_nl(raw: torch.Tensor) -> torch.Tensor:
    b = _blocks(raw, 18)
    d = _f16(b[..., 0:2])
    return _flat(_iq4_nibbles(b[..., 2:18]) * d.unsqueeze(-1))


def dequantize_iq4_xs(raw: torch.Tensor) -> torch.Tensor:
    b = _blocks(raw, 136)
    d = _f16(b[..., 0:2])
    sh = b[..., 2].to(torch.int64) | (b[..., 3].to(torch.int64) << 8)
    sl = b[..., 4:8].to(torch.int64)
    ib = torch.arange(8)
    ls = ((sl[..., ib // 2] >> (4 * (ib % 2))) & 0xF) | (((sh[..., None] >> (2 * ib)) & 3) << 4)
    dl = d.unsqueeze(-1) * (ls.float() - 32.0)                                  # [..., 8]
    qs = b[..., 8:136].reshape(*b.shape[:-1], 8, 16)
    v = _iq4_nibbles(qs) * dl.unsqueeze(-1)                                    # [..., 8, 32]
    return _flat(v.reshape(*b.shape[:-1], 256))


def quantize_fp8_b128(x: torch.Tensor) -> torch.Tensor:
    """[..., K] -> blocks of [f32 multiplier | 128 E4M3 codes]; each block's absmax maps to
    448, the E4M3 maximum."""
    xf = x.float()
    b = xf.reshape(*xf.shape[:-1], xf.shape[-1] // 128, 128)
    s = (b.abs().amax(-1, keepdim=True) / 448.0).clamp_min(1e-12)
    codes = (b / s).to(torch.float8_e4m3fn).view(torch.uint8)
    raw = torch.cat([s.contiguous().view(torch.uint8), codes], -1)
    return raw.reshape(*xf.shape[:-1], -1)


def fp8_b128_from_tiles(codes: torch.Tensor, scale_inv: torch.Tensor, block: int = 128) -> torch.Tensor:
    """A block-scaled fp8 checkpoint tensor (E4M3 codes [N, K], multipliers per block x block
    tile) in the FP8_E4M3_B128 layout, codes unchanged (exact)."""
    N, K = codes.shape
    if K % 128 or block != 128:
        raise ValueError("FP8_E4M3_B128 needs K % 128 == 0 and 128 x 128 tiles")
    s = scale_inv.float().repeat_interleave(block, 0)[:N].reshape(N, K // 128, 1)
    c = codes.contiguous().view(torch.uint8).reshape(N, K // 128, 128)
    return torch.cat([s.contiguous().view(torch.uint8), c], -1).reshape(N, -1)


def dequantize_fp8_b128(raw: torch.Tensor) -> torch.Tensor:
    b = raw.reshape(*raw.shape[:-1], raw.shape[-1] // 132, 132)
    s = b[..., :4].contiguous().view(torch.float32)
    v = b[..., 4:].contiguous().view(torch.float8_e4m3fn).float() * s
    return v.reshape(*raw.shape[:-1], -1)


def _dense(dtype):
    def f(raw: torch.Tensor) -> torch.Tensor:
        n = torch.tensor([], dtype=dtype).element_size()
        return raw.contiguous().view(dtype).float().reshape(*raw.shape[:-1], raw.shape[-1] // n)
    return f


DEQUANT = {
    GGMLType.F32: _dense(torch.float32),
    GGMLType.F16: _dense(torch.float16),
    GGMLType.BF16: _dense(torch.bfloat16),
    GGMLType.Q4_0: dequantize_q4_0,
    GGMLType.Q4_1: dequantize_q4_1,
    GGMLType.Q5_0: dequantize_q5_0,
    GGMLType.Q5_1: dequantize_q5_1,
    GGMLType.Q8_0: dequantize_q8_0,
    GGMLType.Q2_K: dequantize_q2_k,
    GGMLType.Q3_K: dequantize_q3_k,
    GGMLType.Q4_K: dequantize_q4_k,
    GGMLType.Q5_K: dequantize_q5_k,
    GGMLType.Q6_K: dequantize_q6_k,
    GGMLType.Q8_K: dequantize_q8_k,
    GGMLType.IQ4_NL: dequantize_iq4_nl,
    GGMLType.IQ4_XS: dequantize_iq4_xs,
    GGMLType.FP8_E4M3_B128: dequantize_fp8_b128,
}

QUANT = {
    GGMLType.F32: lambda x: x.float().contiguous().view(torch.uint8),
    GGMLType.F16: lambda x: x.half().contiguous().view(torch.uint8),
    GGMLType.BF16: lambda x: x.bfloat16().contiguous().view(torch.uint8),
    GGMLType.Q8_0: quantize_q8_0,
    GGMLType.Q4_K: quantize_q4_k,
    GGMLType.Q6_K: quantize_q6_k,
    GGMLType.FP8_E4M3_B128: quantize_fp8_b128,
}


def dequantize(raw: torch.Tensor, qtype: GGMLType) -> torch.Tensor:
    qtype = GGMLType(qtype)
    if qtype not in DEQUANT:
        from ..quant import extra
        return extra.dequantize(raw, qtype)
    return DEQUANT[qtype](raw)


def quantize(x: torch.Tensor, qtype: GGMLType) -> torch.Tensor:
    qtype = GGMLType(qtype)
    if qtype not in QUANT:
        raise NotImplementedError(f"quantisation to {qtype.name} is not implemented")
    per, _ = BLOCK_GEOMETRY[qtype]
    if x.shape[-1] % per:
        raise ValueError(f"row length {x.shape[-1]} not a multiple of {per} for {qtype.name}")
    return QUANT[qtype](x)
