"""Low-bit GGUF block formats: the IQ lattice formats (IQ1_S, IQ1_M, IQ2_XXS, IQ2_XS, IQ2_S,
IQ3_XXS, IQ3_S), the ternary TQ1_0 / TQ2_0 and the microscaled MXFP4, decoded with torch.

The reference reads these through ``src/iq_quant.rs`` (``dequantize_iq`` with BlockIq1s /
BlockIq2xxs / BlockIq2xs / BlockIq2s / BlockIq3s) and maps ggml type codes with
``ggml_type_to_iq_format`` (``src/iq_quant.rs:493-523``). Its codebooks are placeholders (a
linear 0..7.875 ramp, a 2-bit counting grid), so its output does not match llama.cpp's; here
the formats decode to the same values llama.cpp writes them from.

Every IQ format is "scale x codebook row x sign": a super-block of 256 weights holds one f16
scale, small per-group scale codes, and for each chunk of 4 or 8 weights an index into a
fixed lattice codebook plus sign bits (or, for IQ1, a shared offset of +-1/8). The codebooks
are part of the GGUF format definition; they are taken at run time from the installed
``gguf`` package (``gguf.quants.<TYPE>.grid``), not restated here. 7-bit sign codes expand
to 8 signs whose last sign makes the count of negatives even.

All functions take ``uint8`` tensors whose last dimension holds whole blocks of one row and
return ``float32`` rows; they run on whatever device the input lives on.
"""
from __future__ import annotations

import functools

import torch

from ..gguf.constants import BLOCK_GEOMETRY, GGMLType


# ---------------------------------------------------------------------------- helpers
@functools.lru_cache(maxsize=None)
def _grid_cpu(name: str) -> torch.Tensor:
    try:
        from gguf import quants as gq
    except ImportError as e:          # pragma: no cover - the image ships gguf
        raise RuntimeError(f"{name} needs the lattice codebooks of the 'gguf' package") from e
    cls = getattr(gq, name)
    cls.init_grid()
    rows, width = cls.grid_shape
    return torch.from_numpy(cls.grid.reshape(rows, width).copy()).float()


def grid(name: str, device=None) -> torch.Tensor:
    """Codebook of format ``name`` as float32 [rows, 4 or 8]."""
    g = _grid_cpu(name)
    return g if device is None or torch.device(device).type == "cpu" else g.to(device)


def _even_parity_signs() -> torch.Tensor:
    i = torch.arange(128)
    par = torch.zeros_like(i)
    for b in range(7):
        par ^= (i >> b) & 1
    return i | (par << 7)


_SIGN7 = _even_parity_signs()          # 7-bit code -> 8 sign bits with even parity
_BITS8 = torch.arange(8)


def _sign_bits(byte: torch.Tensor) -> torch.Tensor:
    """[...] integer -> [..., 8] of +1 / -1 (bit j set = element j negative)."""
    return 1.0 - 2.0 * ((byte.unsqueeze(-1) >> _BITS8.to(byte.device)) & 1).float()


def _blocks(raw: torch.Tensor, qtype: GGMLType) -> torch.Tensor:
    if raw.dtype != torch.uint8:
        raise TypeError("raw block tensor must be uint8")
    _, nb = BLOCK_GEOMETRY[qtype]
    if raw.shape[-1] % nb:
        raise ValueError(f"row of {raw.shape[-1]} bytes is not a whole number of {qtype.name} blocks ({nb} B)")
    return raw.reshape(-1, nb)


def _out(v: torch.Tensor, raw: torch.Tensor, qtype: GGMLType) -> torch.Tensor:
    per, nb = BLOCK_GEOMETRY[qtype]
    return v.reshape(*raw.shape[:-1], raw.shape[-1] // nb * per)


def _f16(b: torch.Tensor) -> torch.Tensor:
    return b.contiguous().view(torch.float16).squeeze(-1).float()


def _le(b: torch.Tensor) -> torch.Tensor:
    """Little-endian unsigned integer of the last dim's bytes (up to 4), as int64."""
    b = b.to(torch.int64)
    out = torch.zeros(b.shape[:-1], dtype=torch.int64, device=b.device)
    for k in range(b.shape[-1]):
        out |= b[..., k] << (8 * k)
    return out


# ---------------------------------------------------------------------------- IQ2
def dequantize_iq2_xxs(raw: torch.Tensor) -> torch.Tensor:
    """66 B / 256: f16 d; 8 groups of (4 codebook bytes, u32 = 4 x 7-bit signs | 4-bit scale)."""
    b = _blocks(raw, GGMLType.IQ2_XXS)
    d = _f16(b[:, 0:2])
    g = b[:, 2:].reshape(-1, 8, 8)
    idx = g[..., :4].long()                                       # [n, 8, 4]
    aux = _le(g[..., 4:8])                                        # [n, 8]
    scale = d[:, None] * (0.5 + (aux >> 28).float()) * 0.25
    codes = (aux[..., None] >> (7 * torch.arange(4, device=b.device))) & 127
    sg = _sign_bits(_SIGN7.to(b.device)[codes])                   # [n, 8, 4, 8]
    v = grid("IQ2_XXS", b.device)[idx] * sg * scale[..., None, None]
    return _out(v, raw, GGMLType.IQ2_XXS)


def _nibble_scales(sc: torch.Tensor) -> torch.Tensor:
    """[n, k] bytes -> [n, 2k] 4-bit codes, low nibble first."""
    return torch.stack([sc & 15, sc >> 4], -1).reshape(sc.shape[0], -1).float()


def dequantize_iq2_xs(raw: torch.Tensor) -> torch.Tensor:
    """74 B / 256: f16 d; 32 u16 = 9-bit codebook index | 7-bit sign code; 8 scale bytes
    (one 4-bit scale per 16 weights)."""
    b = _blocks(raw, GGMLType.IQ2_XS)
    d = _f16(b[:, 0:2])
    q = _le(b[:, 2:66].reshape(-1, 32, 2))                        # [n, 32]
    scale = d[:, None] * (0.5 + _nibble_scales(b[:, 66:74].long())) * 0.25      # [n, 16]
    sg = _sign_bits(_SIGN7.to(b.device)[q >> 9])                  # [n, 32, 8]
    v = grid("IQ2_XS", b.device)[q & 511] * sg * scale.repeat_interleave(2, 1)[..., None]
    return _out(v, raw, GGMLType.IQ2_XS)


def dequantize_iq2_s(raw: torch.Tensor) -> torch.Tensor:
    """82 B / 256: f16 d; 32 low index bytes; 32 sign bytes; 8 bytes of 2-bit index highs;
    8 scale bytes (4 bits per 16 weights)."""
    b = _blocks(raw, GGMLType.IQ2_S)
    d = _f16(b[:, 0:2])
    lo = b[:, 2:34].long()
    signs = b[:, 34:66].long()
    qh = b[:, 66:74].long()
    hi = ((qh[..., None] >> (2 * torch.arange(4, device=b.device))) & 3).reshape(-1, 32)
    scale = d[:, None] * (0.5 + _nibble_scales(b[:, 74:82].long())) * 0.25
    v = grid("IQ2_S", b.device)[lo | (hi << 8)] * _sign_bits(signs) * scale.repeat_interleave(2, 1)[..., None]
    return _out(v, raw, GGMLType.IQ2_S)


# ---------------------------------------------------------------------------- IQ3
def dequantize_iq3_xxs(raw: torch.Tensor) -> torch.Tensor:
    """98 B / 256: f16 d; 64 codebook bytes (4 weights each); 8 u32 = 4 x 7-bit signs | scale."""
    b = _blocks(raw, GGMLType.IQ3_XXS)
    d = _f16(b[:, 0:2])
    idx = b[:, 2:66].long().reshape(-1, 8, 8)                     # [n, group, chunk of 4]
    aux = _le(b[:, 66:98].reshape(-1, 8, 4))
    scale = d[:, None] * (0.5 + (aux >> 28).float()) * 0.5
    codes = (aux[..., None] >> (7 * torch.arange(4, device=b.device))) & 127
    sg = _sign_bits(_SIGN7.to(b.device)[codes]).reshape(-1, 8, 8, 4)
    v = grid("IQ3_XXS", b.device)[idx] * sg * scale[..., None, None]
    return _out(v, raw, GGMLType.IQ3_XXS)


def dequantize_iq3_s(raw: torch.Tensor) -> torch.Tensor:
    """110 B / 256: f16 d; 64 low index bytes; 8 bytes of 1-bit index highs; 32 sign bytes;
    4 scale bytes (odd scales 1 + 2s per 32 weights)."""
    b = _blocks(raw, GGMLType.IQ3_S)
    d = _f16(b[:, 0:2])
    lo = b[:, 2:66].long()
    hi = ((b[:, 66:74].long()[..., None] >> _BITS8.to(b.device)) & 1).reshape(-1, 64)
    sg = _sign_bits(b[:, 74:106].long()).reshape(-1, 64, 4)
    scale = d[:, None] * (1.0 + 2.0 * _nibble_scales(b[:, 106:110].long()))       # [n, 8]
    v = grid("IQ3_S", b.device)[lo | (hi << 8)] * sg * scale.repeat_interleave(8, 1)[..., None]
    return _out(v, raw, GGMLType.IQ3_S)


# ---------------------------------------------------------------------------- IQ1
IQ1_DELTA = 0.125


def dequantize_iq1_s(raw: torch.Tensor) -> torch.Tensor:
    """50 B / 256: f16 d; 32 low index bytes; 8 u16 = 4 x 3-bit index highs | 3-bit scale |
    offset sign. Weight = d (2s + 1) (grid + -1/8)."""
    b = _blocks(raw, GGMLType.IQ1_S)
    d = _f16(b[:, 0:2])
    lo = b[:, 2:34].long().reshape(-1, 8, 4)
    qh = _le(b[:, 34:50].reshape(-1, 8, 2))                       # [n, 8]
    hi = (qh[..., None] >> (3 * torch.arange(4, device=b.device))) & 7
    dl = d[:, None] * (2.0 * ((qh >> 12) & 7).float() + 1.0)
    delta = torch.where((qh & 0x8000) != 0, -IQ1_DELTA, IQ1_DELTA)
    v = dl[..., None, None] * (grid("IQ1_S", b.device)[lo | (hi << 8)] + delta[..., None, None])
    return _out(v, raw, GGMLType.IQ1_S)


def dequantize_iq1_m(raw: torch.Tensor) -> torch.Tensor:
    """56 B / 256: 32 low index bytes; 16 bytes of (3-bit index high | offset sign) nibbles;
    4 u16 holding 16 x 3-bit scales in their low 12 bits and the f16 d in their top nibbles."""
    b = _blocks(raw, GGMLType.IQ1_M)
    lo = b[:, 0:32].long()                                        # [n, 32 chunks of 8]
    nib = torch.stack([b[:, 32:48].long() & 15, b[:, 32:48].long() >> 4], -1).reshape(-1, 32)
    s = _le(b[:, 48:56].reshape(-1, 4, 2))                        # [n, 4]
    dbits = ((s >> 12) << (4 * torch.arange(4, device=b.device))).sum(-1)
    d = (dbits - ((dbits >> 15) << 16)).to(torch.int16).view(torch.float16).float()   # the f16's bits
    sc = ((s[..., None] >> (3 * torch.arange(4, device=b.device))) & 7).reshape(-1, 16)
    dl = d[:, None] * (2.0 * sc.float() + 1.0)                    # [n, 16], two chunks each
    delta = torch.where((nib & 8) != 0, -IQ1_DELTA, IQ1_DELTA)
    v = (grid("IQ1_M", b.device)[lo | ((nib & 7) << 8)] + delta[..., None]) * dl.repeat_interleave(2, 1)[..., None]
    return _out(v, raw, GGMLType.IQ1_M)


# ---------------------------------------------------------------------------- ternary / fp4
_POW3 = torch.tensor([1, 3, 9, 27, 81])


def _trits(byte: torch.Tensor, n: int) -> torch.Tensor:
    """Base-3 digits stored as fixed-point fractions: digit k of byte b is
    ((b * 3^k mod 256) * 3) >> 8. [..., m] -> [..., n, m] in {0, 1, 2}."""
    p = _POW3[:n].to(byte.device)
    return (((byte[..., None, :] * p[:, None]) & 255) * 3) >> 8


def dequantize_tq1_0(raw: torch.Tensor) -> torch.Tensor:
    """54 B / 256 (1.69 bits): 48 bytes of five trits, 4 bytes of four trits, f16 d."""
    b = _blocks(raw, GGMLType.TQ1_0)
    q = b[:, :52].long()
    t = torch.cat([_trits(q[:, 0:32], 5).reshape(-1, 160), _trits(q[:, 32:48], 5).reshape(-1, 80),
                   _trits(q[:, 48:52], 4).reshape(-1, 16)], 1)
    v = (t - 1).float() * _f16(b[:, 52:54])[:, None]
    return _out(v, raw, GGMLType.TQ1_0)


def dequantize_tq2_0(raw: torch.Tensor) -> torch.Tensor:
    """66 B / 256: 64 bytes of four 2-bit codes (code - 1 in {-1, 0, 1}), f16 d."""
    b = _blocks(raw, GGMLType.TQ2_0)
    q = b[:, :64].long().reshape(-1, 2, 1, 32)
    t = (q >> (2 * torch.arange(4, device=b.device)).reshape(1, 1, 4, 1)) & 3
    v = (t.reshape(-1, 256) - 1).float() * _f16(b[:, 64:66])[:, None]
    return _out(v, raw, GGMLType.TQ2_0)


E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0])


def dequantize_mxfp4(raw: torch.Tensor) -> torch.Tensor:
    """17 B / 32 (OCP MX): E8M0 shared exponent (2^(e - 127)), 16 bytes of E2M1 nibbles
    (elements 0..15 in the low nibbles, 16..31 in the high)."""
    b = _blocks(raw, GGMLType.MXFP4)
    scale = torch.ldexp(torch.ones(b.shape[0], device=b.device), b[:, 0].long() - 127)
    q = b[:, 1:17].long()
    v = E2M1.to(b.device)[torch.cat([q & 15, q >> 4], 1)] * scale[:, None]
    return _out(v, raw, GGMLType.MXFP4)


DEQUANT = {
    GGMLType.IQ2_XXS: dequantize_iq2_xxs,
    GGMLType.IQ2_XS: dequantize_iq2_xs,
    GGMLType.IQ2_S: dequantize_iq2_s,
    GGMLType.IQ3_XXS: dequantize_iq3_xxs,
    GGMLType.IQ3_S: dequantize_iq3_s,
    GGMLType.IQ1_S: dequantize_iq1_s,
    GGMLType.IQ1_M: dequantize_iq1_m,
    GGMLType.TQ1_0: dequantize_tq1_0,
    GGMLType.TQ2_0: dequantize_tq2_0,
    GGMLType.MXFP4: dequantize_mxfp4,
}


def dequantize(raw: torch.Tensor, qtype: GGMLType) -> torch.Tensor:
    qtype = GGMLType(qtype)
    fn = DEQUANT.get(qtype)
    if fn is None:
        raise NotImplementedError(f"dequantisation of {qtype.name} is not implemented")
    return fn(raw)


def iq_format_of(ggml_type: int) -> GGMLType | None:
    """The low-bit format of a ggml type code, None for the other formats (the reference's
    ``ggml_type_to_iq_format``, with ggml's own type codes)."""
    try:
        t = GGMLType(ggml_type)
    except ValueError:
        return None
    return t if t in DEQUANT or t in (GGMLType.IQ4_NL, GGMLType.IQ4_XS) else None
