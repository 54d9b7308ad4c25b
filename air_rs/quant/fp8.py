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
