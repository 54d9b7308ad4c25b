"""GEMM entry point of the prefill / large-batch path.

``linear`` runs the tcgen05 dequant-fused GEMM (``air_rs._C.gemm_q``) when it supports the
weight format and shape; the ``baseline`` implementation (dequantise the weight to a bf16
scratch with our kernel, then a library matmul) exists only as the comparison arm and for
formats the fused kernel does not cover yet.
"""
from __future__ import annotations

import os

import torch

from . import QWeight, require_ext, FMT_BF16, count_launch

_FORCE_BASELINE = os.environ.get("AIR_GEMM_IMPL", "") == "baseline"


def tc_supported(w: QWeight, T: int) -> bool:
    ext = require_ext()
    return hasattr(ext, "gemm_q") and not _FORCE_BASELINE and w.K % 256 == 0 and w.N % 128 == 0


def linear(x: torch.Tensor, w: QWeight, out: torch.Tensor, runner=None) -> torch.Tensor:
    T = x.shape[0]
    if tc_supported(w, T):
        ext = require_ext()
        ext.gemm_q(w.fmt, w.data, w.scales, w.row_bytes, w.N, w.K, x, out)
        count_launch()
        return out
    return linear_baseline(x, w, out, runner)


def linear_baseline(x: torch.Tensor, w: QWeight, out: torch.Tensor, runner=None) -> torch.Tensor:
    if w.fmt == FMT_BF16:
        wt = w.data
    else:
        scratch = getattr(runner, "_wscratch", None) if runner is not None else None
        need = w.N * w.K
        if scratch is None or scratch.numel() < need:
            scratch = torch.empty(need, dtype=torch.bfloat16, device=x.device)
            if runner is not None:
                runner._wscratch = scratch
        wt = scratch[:need].view(w.N, w.K)
        w.dequantize_bf16(wt)
    if out.dtype == torch.bfloat16:
        torch.matmul(x, wt.t(), out=out)
    else:
        out.copy_(torch.matmul(x, wt.t()))
    return out
