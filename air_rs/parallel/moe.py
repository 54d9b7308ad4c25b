"""Mixture-of-experts FFN (placeholder until the fused EP path lands)."""


def moe_ffn_decode(runner, lw, B, x, xq, xds):
    raise NotImplementedError("MoE FFN")


def moe_ffn_gemm(runner, lw, B, x):
    raise NotImplementedError("MoE FFN")


def moe_ffn_prefill(runner, lw, T, x, xn):
    raise NotImplementedError("MoE FFN")
