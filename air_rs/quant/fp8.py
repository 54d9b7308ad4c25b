"""FP8 E4M3 (OCP "fn": no infinities, max 448) and E5M2 (IEEE-like, max 57344) codecs with
round-to-nearest-even and saturation (reference ``src/fp8.rs``), plus a per-tensor-scaled
FP8 linear layer. Bit-for-bit equal to ``torch.float8_e4m3fn`` / ``torch.float8_e5m2``
conversions for finite inputs within range (tested).
"""
from __future__ import annotations

import torch

E4M3_MAX = 448.0
E5M2_MAX = 57344.0


def _encode(x: torch.Tensor, exp_bits: int, man_bits: int, bias: int, max_val: float, fn: bool) -> torch.Tensor:
    x = x.float()
    sign = (x < 0) | ((x == 0) & (torch.signbit(x)))
    a = x.abs()
    nan = torch.isnan(x)
    a = torch.clamp(a, max=max_val)                       # saturate (finite formats)
    # exponent of a (normal range); subnormals share the minimum exponent
    min_exp = 1 - bias
    e = torch.floor(torch.log2(torch.where(a > 0, a, torch.ones_like(a))))
    e = torch.clamp(e, min=min_exp)
    step = torch.exp2(e - man_bits)                       # spacing at this exponent
    q = torch.round(a / step)                             # round half to even
    # rounding up can carry into the next binade
    carry = q >= 2 ** (man_bits + 1)
    e = torch.where(carry, e + 1, e)
    q = torch.where(carry, q / 2, q)
    is_sub = (q < 2 ** man_bits)                          # no implicit bit
    exp_field = torch.where(is_sub, torch.zeros_like(e), e + bias)
    man_field = torch.where(is_sub, q, q - 2 ** man_bits)
    bits = (exp_field.to(torch.int32) << man_bits) | man_field.to(torch.int32)
    top = (1 << (exp_bits + man_bits)) - 1
    if fn:
        bits = torch.where(nan, torch.full_like(bits, top), bits)   # S.1111.111 is the only NaN
    else:
        bits = torch.where(nan, torch.full_like(bits, top - (1 << man_bits) + 2), bits)
    bits = bits | (sign.to(torch.int32) << (exp_bits + man_bits))
    return bits.to(torch.uint8)


def _decode(b: torch.Tensor, exp_bits: int, man_bits: int, bias: int, fn: bool) -> torch.Tensor:
    b = b.to(torch.int32)
    s = torch.where((b >> (exp_bits + man_bits)) & 1 == 1, -1.0, 1.0)
    ef = (b >> man_bits) & ((1 << exp_bits) - 1)
    mf = (b & ((1 << man_bits) - 1)).float()
    sub = ef == 0
    val = torch.where(sub, mf * 2.0 ** (1 - bias - man_bits),
                      (1 + mf / 2 ** man_bits) * torch.exp2(ef.float() - bias))
    if fn:
        nan = (ef == (1 << exp_bits) - 1) & (mf == (1 << man_bits) - 1)
    else:
        nan = (ef == (1 << exp_bits) - 1) & (mf != 0)
        val = torch.where((ef == (1 << exp_bits) - 1) & (mf == 0), torch.full_like(val, float("inf")), val)
    return torch.where(nan, torch.full_like(val, float("nan")), s * val)


def e4m3_from_f32(x):
    return _encode(torch.as_tensor(x), 4, 3, 7, E4M3_MAX, True)


def e4m3_to_f32(b):
    return _decode(torch.as_tensor(b), 4, 3, 7, True)


def e5m2_from_f32(x):
    return _encode(torch.as_tensor(x), 5, 2, 15, E5M2_MAX, False)


def e5m2_to_f32(b):
    return _decode(torch.as_tensor(b), 5, 2, 15, False)


class Fp8Linear:
    """y = x @ (scale * W_fp8)^T with one scale per tensor (amax / 448)."""

    def __init__(self, w: torch.Tensor):
        amax = float(w.abs().max()) or 1.0
        self.scale = amax / E4M3_MAX
        self.codes = e4m3_from_f32(w / self.scale)
        self.shape = tuple(w.shape)

    def dequantize(self) -> torch.Tensor:
        return e4m3_to_f32(self.codes) * self.scale

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return x.float() @ self.dequantize().t()


# ---------------------------------------------------------------------------- block-scaled fp8
FP8_BLOCK = 128


def block_quantize_fp8(w: torch.Tensor, block: int = FP8_BLOCK) -> tuple[torch.Tensor, torch.Tensor]:
    """W [N, K] -> (E4M3 codes [N, K] as torch.float8_e4m3fn, inverse scales [ceil(N/b), ceil(K/b)]):
    each block x block tile is scaled so its absmax maps to 448 (the E4M3 maximum); the stored
    scale is the multiplier that restores the tile (the ``weight_scale_inv`` convention of
    block-scaled fp8 checkpoints)."""
    N, K = w.shape
    nb, kb = -(-N // block), -(-K // block)
    wp = torch.nn.functional.pad(w.float(), (0, kb * block - K, 0, nb * block - N))
    tiles = wp.reshape(nb, block, kb, block)
    amax = tiles.abs().amax((1, 3)).clamp_min(1e-12)
    scale_inv = amax / 448.0
    q = (tiles / scale_inv[:, None, :, None]).reshape(nb * block, kb * block)[:N, :K]
    return q.to(torch.float8_e4m3fn), scale_inv


def block_dequantize_fp8(q: torch.Tensor, scale_inv: torch.Tensor, block: int = FP8_BLOCK) -> torch.Tensor:
    """Inverse of ``block_quantize_fp8``: codes [N, K] times the tile scale -> fp32."""
    N, K = q.shape
    s = scale_inv.float().repeat_interleave(block, 0)[:N].repeat_interleave(block, 1)[:, :K]
    return q.float() * s
