"""Mixture-of-experts FFN on the GPU runner (reference ``src/moe.rs:163-300``).

Routing runs on the device (``moe_route``: fp32 router logits, softmax, top-k, renormalise)
and produces a dense combine matrix ``cw[T, E]`` (zero for experts a token did not pick), so
the step stays CUDA-graph capturable with no host round trip. Each expert's SwiGLU FFN then
runs over the batch with the runner's own kernels (decode GEMV with the fused SwiGLU
epilogue, or the tcgen05 GEMM path) and ``moe_combine`` adds ``cw[:, e] * y_e`` into the
residual stream; rows whose weight is zero are skipped there. Every expert's weights are
streamed once per step — for large batches (the Mixtral config's 128-sequence decode) every
expert is active anyway.
"""
from __future__ import annotations

import torch

from .. import ops


def _ensure(rn, name, shape, dtype):
    t = getattr(rn, name, None)
    if t is None or t.shape[0] < shape[0] or tuple(t.shape[1:]) != tuple(shape[1:]):
        if torch.cuda.is_available() and torch.cuda.is_current_stream_capturing():
            raise RuntimeError(f"MoE buffer {name} must be allocated before CUDA-graph capture")
        t = torch.zeros(shape, dtype=dtype, device=rn.device)
        setattr(rn, name, t)
    return t


def _check(rn):
    if rn.tp_size > 1:
        raise NotImplementedError("MoE layers under tensor parallelism: use expert parallelism")


def moe_ffn_decode(rn, lw, B, x, xq, xds):
    """GEMV path (B <= 8). Expects ``rn.xn_b[:B]`` = normalised input (bf16) and xq/xds its
    quantised form."""
    _check(rn)
    ext = ops.require_ext()
    E = len(lw.experts_gu)
    cw = _ensure(rn, "moe_cw", (rn.max_batch, E), torch.float32)
    hq = _ensure(rn, "moe_hq", (rn.max_batch, rn.Fp), torch.int8)
    hds = _ensure(rn, "moe_hds", (rn.max_batch, rn.Fp // 32, 2), torch.float32)
    ext.moe_route(rn.xn_b[:B], B, lw.router, rn.cfg.moe_top_k, True, cw[:B], None, None)
    ops.count_launch()
    for e in range(E):
        gu, dn = lw.experts_gu[e], lw.experts_down[e]
        ops.gemv(gu.part(0), xq, xds, B, ops.EPI_SWIGLU, w2=gu.part(1), out_f32=rn.h[:B], ld_out=rn.Fp)
        ops.rmsnorm_quant(rn.h[:B], None, 0.0, hq[:B], hds[:B])
        ops.gemv(dn, hq[:B], hds[:B], B, ops.EPI_STORE, out_f32=rn.y[:B])
        ext.moe_combine(x[:B], rn.y[:B], cw[:B], e, E, B)
        ops.count_launch()


def _ffn_tokens(rn, lw, T, x, xn, gu_buf, h_buf, y_buf, cw):
    ext = ops.require_ext()
    E = len(lw.experts_gu)
    ext.moe_route(xn[:T], T, lw.router, rn.cfg.moe_top_k, True, cw[:T], None, None)
    ops.count_launch()
    for e in range(E):
        gu, dn = lw.experts_gu[e], lw.experts_down[e]
        rn.linear(xn[:T], gu, gu_buf[:T])
        ops.swiglu(gu_buf[:T], T, rn.F, out_bf16=h_buf[:T], ld_out=rn.Fp, up_off=gu.parts[1][0])
        rn.linear(h_buf[:T], dn, y_buf[:T])
        ext.moe_combine(x[:T], y_buf[:T], cw[:T], e, E, T)
        ops.count_launch()


def moe_ffn_gemm(rn, lw, B, x):
    """Batched decode (GEMM path): input is ``rn.xn_b[:B]`` (bf16, normalised)."""
    _check(rn)
    E = len(lw.experts_gu)
    cw = _ensure(rn, "moe_cw", (rn.max_batch, E), torch.float32)
    _ffn_tokens(rn, lw, B, x, rn.xn_b, rn.gu_b, rn.h_b, rn.y, cw)


def moe_ffn_prefill(rn, lw, T, x, xn):
    _check(rn)
    E = len(lw.experts_gu)
    cw = rn._ws("moe_cw", (T, E), torch.float32)
    gu = rn._ws("gu", (T, rn.gu_w), torch.bfloat16)
    hb = rn._ws("hb", (T, rn.Fp), torch.bfloat16, zero=True)
    y = rn._ws("moe_y", (T, rn.H), torch.float32)
    _ffn_tokens(rn, lw, T, x, xn, gu, hb, y, cw)
