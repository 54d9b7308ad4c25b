"""Mixture-of-experts FFN on the GPU runner, with expert parallelism (reference
``src/moe.rs:163-300`` routing + per-token expert loop, ``src/moe.rs:510-536`` EP router).

Routing runs on the device (``moe_route``: fp32 router logits, softmax, top-k, renormalise)
into a dense combine matrix ``cw[T, E]`` (zero for experts a token did not pick), so the step
has no host round trip and stays CUDA-graph capturable.

* Decode GEMV path (B <= 8): each local expert's SwiGLU FFN runs over the batch with the
  fused GEMV kernels (weights are read once either way) and ``moe_combine`` adds
  ``cw[:, e] * y_e`` (zero-weight rows skipped).
* Batched / prefill path: up to eight local experts at a time, ``moe_select_grouped`` lists
  each expert's tokens, ``moe_gather_grouped`` packs their rows into one buffer (expert g at
  rows g*T..), ONE grouped tcgen05 GEMM runs gate|up for every expert of the group and one
  runs down (token tiles past an expert's device-side count exit at once — fixed launch
  shapes, graph capturable), SwiGLU runs over the packed rows, and ``moe_scatter_grouped``
  adds each token's weighted expert outputs in expert order. Per-expert launches remain for
  host-resident experts (expert cache) and formats without a tensor-core kernel.

Expert parallelism: under TP the experts are spread over the ranks (expert e on rank
e % tp) while attention stays tensor parallel, so every rank holds every token's
activations after the attention all-reduce — the dispatch is a local gather with no
communication, and the combine is the sum over ranks of each rank's partial expert output,
done by the same fused peer-memory push / reduce-RMSNorm as the dense row-parallel layers
(NCCL all-reduce when the peer path is off).
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


def _ids(lw):
    return lw.expert_ids or list(range(len(lw.experts_gu)))


def _experts(rn, lw, cw, T):
    """(gate|up, down, global id) of this rank's experts: all of them, or — with host-resident
    experts behind an expert cache — only those some token picked, made resident on demand."""
    cache = getattr(rn, "expert_cache", None)
    if cache is None:
        return zip(lw.experts_gu, lw.experts_down, _ids(lw))
    return cache.experts_for(lw, (cw[:T] > 0).any(0).cpu())


def _finish(rn, T, x, partial, peer):
    """EP combine: partial expert outputs of this rank -> every rank's residual stream."""
    if rn.tp_size == 1:
        return
    if peer is not None:
        peer.push(partial[:T], T)            # summed by the next reduce-RMSNorm
    else:
        rn.tp.all_reduce_add(partial[:T], x[:T])


def moe_ffn_decode(rn, lw, B, x, xq, xds, peer=None):
    """GEMV path (B <= 8). Expects ``rn.xn_b[:B]`` = normalised input (bf16) and xq/xds its
    quantised form. With resident tensor-core experts the grouped GEMM path runs instead:
    experts no token picked exit before reading a byte of their weights (a per-expert GEMV
    chain would stream every expert), so a batch-1 step reads top_k of n_experts."""
    if _grouped_ok(rn, lw):
        moe_ffn_gemm(rn, lw, B, x, peer)
        return
    ext = ops.require_ext()
    E = rn.cfg.n_experts
    cw = _ensure(rn, "moe_cw", (rn.max_batch, E), torch.float32)
    hq = _ensure(rn, "moe_hq", (rn.max_batch, rn.Fp), torch.int8)
    hds = _ensure(rn, "moe_hds", (rn.max_batch, rn.Fp // 32, 2), torch.float32)
    ext.moe_route(rn.xn_b[:B], B, lw.router, rn.cfg.moe_top_k, True, cw[:B], None, None)
    ops.count_launch()
    ep = rn.tp_size > 1
    acc = x
    if ep:
        acc = _ensure(rn, "moe_part", (rn.max_batch, rn.H), torch.float32)
        acc[:B].zero_()
    for gu, dn, e in _experts(rn, lw, cw, B):
        ops.gemv(gu.part(0), xq, xds, B, ops.EPI_SWIGLU, w2=gu.part(1), out_f32=rn.h[:B], ld_out=rn.Fp)
        ops.rmsnorm_quant(rn.h[:B], None, 0.0, hq[:B], hds[:B])
        ops.gemv(dn, hq[:B], hds[:B], B, ops.EPI_STORE, out_f32=rn.y[:B])
        ext.moe_combine(acc[:B], rn.y[:B], cw[:B], e, E, B)
        ops.count_launch()
    if ep:
        _finish(rn, B, x, acc, peer)


GROUP = 8      # experts per grouped launch (the GEMM's group limit)


def _grouped_ok(rn, lw) -> bool:
    """All local experts resident and on the tensor-core GEMM: one launch per group of 8."""
    import os
    from ..ops import gemm
    if getattr(rn, "expert_cache", None) is not None or os.environ.get("AIR_MOE_GROUPED", "1") == "0":
        return False
    ws = list(lw.experts_gu) + list(lw.experts_down)
    return bool(ws) and all(gemm.tc_supported(w) for w in ws)


def _ffn_tokens_grouped(rn, lw, T, x, xn, cw, acc, alloc, prefix):
    """Routed experts in groups of up to GROUP: grouped select / gather, one grouped GEMM for
    gate|up and one for down over every expert of the group, SwiGLU over the packed rows, and
    a grouped scatter that adds each token's expert outputs in a fixed order."""
    from ..ops import gemm
    ext = ops.require_ext()
    ids = _ids(lw)
    gid_cache = getattr(lw, "_group_ids", None)
    if gid_cache is None:
        if torch.cuda.is_available() and torch.cuda.is_current_stream_capturing():
            raise RuntimeError("MoE group ids must be staged before CUDA-graph capture")
        gid_cache = lw._group_ids = [torch.tensor(ids[i:i + GROUP], dtype=torch.int32, device=rn.device)
                                     for i in range(0, len(ids), GROUP)]
    G = min(GROUP, len(ids))
    # decode buffers are sized once for the largest batch (a captured graph keeps pointers)
    cap = rn.max_batch if prefix == "moe_d_" else T
    idx = alloc(prefix + "gidx", (G * cap,), torch.int32)
    wts = alloc(prefix + "gwts", (G * cap,), torch.float32)
    pos = alloc(prefix + "gpos", (G * cap,), torch.int32)
    cnt = alloc(prefix + "gcnt", (G,), torch.int32)
    xg = alloc(prefix + "gxg", (G * cap, rn.H), torch.bfloat16)
    gu_buf = alloc(prefix + "ggu", (G * cap, rn.gu_w), torch.bfloat16)
    h_buf = alloc(prefix + "gh", (G * cap, rn.Fp), torch.bfloat16)
    y_buf = alloc(prefix + "gy", (G * cap, rn.H), torch.float32)
    up_off = lw.experts_gu[0].parts[1][0]
    for c, gids in enumerate(gid_cache):
        g = gids.numel()
        gu_w = lw.experts_gu[c * GROUP:c * GROUP + g]
        dn_w = lw.experts_down[c * GROUP:c * GROUP + g]
        ext.moe_select_grouped(cw[:T], gids, T, idx, wts, cnt, pos)
        ext.moe_gather_grouped(xn[:T], idx, cnt, g, T, xg)
        gemm.linear_grouped(xg, gu_w, gu_buf, cnt, T, err=rn.err)
        ops.swiglu(gu_buf[:g * T], g * T, rn.F, out_bf16=h_buf[:g * T], ld_out=rn.Fp, up_off=up_off, act=rn.act)
        gemm.linear_grouped(h_buf, dn_w, y_buf, cnt, T, err=rn.err)
        ext.moe_scatter_grouped(acc[:T], y_buf, pos, wts, g, T)
        ops.count_launch(3)


def _ffn_tokens(rn, lw, T, x, xn, bufs, peer=None, alloc=None, prefix=""):
    ext = ops.require_ext()
    E = rn.cfg.n_experts
    cw, idx, wts, cnt, xg, gu_buf, h_buf, y_buf = (bufs[k] for k in ("cw", "idx", "wts", "cnt", "xg", "gu", "h", "y"))
    ext.moe_route(xn[:T], T, lw.router, rn.cfg.moe_top_k, True, cw[:T], None, None)
    ops.count_launch()
    ep = rn.tp_size > 1
    acc = bufs["part"] if ep else x
    if ep:
        acc[:T].zero_()
    if alloc is not None and _grouped_ok(rn, lw):
        _ffn_tokens_grouped(rn, lw, T, x, xn, cw, acc, alloc, prefix)
        if ep:
            _finish(rn, T, x, acc, peer)
        return
    for j, (gu, dn, e) in enumerate(_experts(rn, lw, cw, T)):
        c = cnt[j:j + 1]
        ext.moe_select(cw[:T], e, T, idx, wts, c)
        ext.moe_gather(xn[:T], idx, c, T, xg)
        rn.linear_rows(xg[:T], gu, gu_buf[:T], c)
        ops.swiglu(gu_buf[:T], T, rn.F, out_bf16=h_buf[:T], ld_out=rn.Fp, up_off=gu.parts[1][0])
        rn.linear_rows(h_buf[:T], dn, y_buf[:T], c)
        ext.moe_scatter(acc[:T], y_buf[:T], idx, wts, c, T)
        ops.count_launch(3)
    if ep:
        _finish(rn, T, x, acc, peer)


def _bufs(rn, T, prefix, alloc):
    E = rn.cfg.n_experts
    return {"cw": alloc(prefix + "cw", (T, E), torch.float32),
            "idx": alloc(prefix + "idx", (T,), torch.int32),
            "wts": alloc(prefix + "wts", (T,), torch.float32),
            "cnt": alloc(prefix + "cnt", (max(1, len(rn.w.layers[0].experts_gu)),), torch.int32),
            "xg": alloc(prefix + "xg", (T, rn.H), torch.bfloat16),
            "gu": alloc(prefix + "gu", (T, rn.gu_w), torch.bfloat16),
            "h": alloc(prefix + "h", (T, rn.Fp), torch.bfloat16),
            "y": alloc(prefix + "y", (T, rn.H), torch.float32),
            "part": alloc(prefix + "part", (T, rn.H), torch.float32)}


def moe_ffn_gemm(rn, lw, B, x, peer=None):
    """Batched decode (GEMM path): input is ``rn.xn_b[:B]`` (bf16, normalised)."""
    alloc = lambda n, s, d: _ensure(rn, n, s, d)
    bufs = _bufs(rn, rn.max_batch, "moe_d_", alloc)
    _ffn_tokens(rn, lw, B, x, rn.xn_b, bufs, peer, alloc=alloc, prefix="moe_d_")


def moe_ffn_prefill(rn, lw, T, x, xn):
    alloc = lambda n, s, d: rn._ws(n, s, d, zero=(n.endswith("h")))
    bufs = _bufs(rn, T, "moe_p_", alloc)
    _ffn_tokens(rn, lw, T, x, xn, bufs, None, alloc=alloc, prefix="moe_p_")
