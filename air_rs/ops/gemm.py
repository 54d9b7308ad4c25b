"""GEMM entry point of the prefill / large-batch path.

``linear`` runs the tcgen05 dequant-fused GEMM (``air_rs._C.gemm_q``) for Q4_K, Q8_0,
block-scaled FP8 and bf16 weights; split-K partials go to a per-device workspace owned here (allocated once, before
any CUDA-graph capture, and grown only outside capture). The ``baseline`` implementation
(dequantise to a bf16 scratch with our kernel, then a library matmul) exists as the
comparison arm (``AIR_GEMM_IMPL=baseline``) and for formats without a fused kernel.
"""
from __future__ import annotations

import os

import torch

from . import QWeight, require_ext, FMT_BF16, FMT_FP8, FMT_Q4K, FMT_Q8_0, count_launch

GEMM_STORE_F32, GEMM_STORE_BF16, GEMM_RESIDUAL, GEMM_PEER_PUSH = 0, 1, 2, 3


def _baseline_forced() -> bool:
    return os.environ.get("AIR_GEMM_IMPL", "") == "baseline"


def tc_supported(w: QWeight) -> bool:
    if _baseline_forced():
        return False
    if w.fmt == FMT_Q4K:
        return w.K % 256 == 0 and w.data.dim() == 4
    if w.fmt == FMT_BF16:
        return w.K % 64 == 0
    if w.fmt == FMT_FP8:
        return w.K % 256 == 0 and w.scales is not None
    if w.fmt == FMT_Q8_0:
        # int8 codes + f16 block scales fed by TMA; the scale rows must be 16-byte strides
        return w.K % 256 == 0 and w.scales is not None and os.environ.get("AIR_GEMM_Q8", "1") != "0"
    return False


class _Workspace:
    """Split-K scratch for one device: fp32 partials + self-resetting tile counters."""

    def __init__(self, device):
        self.device = device
        self.ws = torch.zeros(0, dtype=torch.float32, device=device)
        self.cnt = torch.zeros(0, dtype=torch.int32, device=device)
        # error word for callers that pass none (bounded waits report into it)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)

    def ensure(self, floats: int, counters: int):
        if self.ws.numel() < floats:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("gemm workspace must be sized before CUDA-graph capture")
            self.ws = torch.zeros(max(floats, 2 * self.ws.numel()), dtype=torch.float32, device=self.device)
        if self.cnt.numel() < counters:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("gemm counters must be sized before CUDA-graph capture")
            self.cnt = torch.zeros(max(counters, 2 * self.cnt.numel(), 1024), dtype=torch.int32,
                                   device=self.device)
        return self.ws, self.cnt


_WS: dict = {}


def workspace(device) -> _Workspace:
    key = torch.device(device)
    w = _WS.get(key)
    if w is None:
        w = _WS[key] = _Workspace(key)
    return w


def linear(x: torch.Tensor, w: QWeight, out: torch.Tensor, runner=None, *, residual: bool = False,
           splits: int | None = None, err: torch.Tensor | None = None,
           dbg: torch.Tensor | None = None, row_count: torch.Tensor | None = None,
           push_meta: torch.Tensor | None = None) -> torch.Tensor:
    """out = x @ W^T (or out += x @ W^T when residual, out fp32). ``row_count`` (device int32)
    limits the tensor-core path to the first rows (token tiles past it exit at once).
    ``push_meta`` (a ``PeerComm`` push table): the epilogue stores the result into the
    tensor-parallel peer receive buffers instead of ``out`` (tensor-core path only)."""
    T = x.shape[0]
    if T == 0:
        return out
    if w.fmt == FMT_FP8 and push_meta is None and row_count is None and fp8_mma_enabled() and w.K % 128 == 0:
        return linear_fp8(x, w, out, residual=residual, splits=splits, err=err)
    if tc_supported(w):
        ext = require_ext()
        if push_meta is not None:
            mode = GEMM_PEER_PUSH
        elif residual:
            mode = GEMM_RESIDUAL
        else:
            mode = GEMM_STORE_BF16 if out.dtype == torch.bfloat16 else GEMM_STORE_F32
        s = splits if splits is not None else ext.gemm_q_splits(w.N, w.K, T, w.fmt)
        ws = cnt = None
        if s > 1:
            ws, cnt = workspace(x.device).ensure(ext.gemm_q_workspace(w.N, w.K, T, w.fmt, s),
                                                 ext.gemm_q_counters(w.N, T))
        if err is None:
            err = workspace(x.device).err
        ext.gemm_q(w.fmt, w.data, w.scales, w.row_bytes, w.N, w.K, x, out, mode, s, ws, cnt, err, dbg, row_count,
                   push_meta)
        count_launch()
        return out
    if push_meta is not None:
        raise ValueError("peer-push GEMM epilogue needs the tensor-core path")
    if residual:
        tmp = linear_baseline(x, w, torch.empty(T, w.N, dtype=torch.float32, device=x.device), runner)
        out.add_(tmp)
        return out
    return linear_baseline(x, w, out, runner)


def fp8_mma_enabled() -> bool:
    """Block-scaled FP8 weights run the W8A8 kernel by default (activations quantised to E4M3
    with one scale per token, ``kind::f8f6f4`` MMAs; 1.1-1.8x faster than dequantising the
    weights at every measured Llama-3-8B shape, T = 16..512). AIR_FP8_MMA=0 keeps bf16
    activations: the weights are then dequantised to bf16 inside the tensor-core GEMM."""
    return os.environ.get("AIR_FP8_MMA", "1") != "0" and not _baseline_forced()


def quant_fp8_rows(x: torch.Tensor):
    """bf16 rows -> (E4M3 codes [T, K] uint8, f32 scale per row [T]); scale = row amax / 448."""
    T, K = x.shape
    xq = torch.empty(T, K, dtype=torch.uint8, device=x.device)
    xs = torch.empty(T, dtype=torch.float32, device=x.device)
    require_ext().quant_fp8_rows(x, xq, xs)
    count_launch()
    return xq, xs


def linear_fp8(x: torch.Tensor, w: QWeight, out: torch.Tensor, *, residual: bool = False,
               splits: int | None = None, err: torch.Tensor | None = None) -> torch.Tensor:
    """W8A8 FP8 GEMM: out (+)= dequant(quant_fp8(x)) @ dequant(W)^T on the tensor cores; the
    weights' per-128-block multipliers are applied per K block in f32, the activations' per-token
    scale in the epilogue (reference src/fp8.rs:28-310,
    src/w8a8.rs:40-160)."""
    if w.fmt != FMT_FP8 or w.scales is None:
        raise ValueError("linear_fp8 needs block-scaled FP8 weights")
    ext = require_ext()
    T = x.shape[0]
    xq, xs = quant_fp8_rows(x)
    mode = GEMM_RESIDUAL if residual else (GEMM_STORE_BF16 if out.dtype == torch.bfloat16 else GEMM_STORE_F32)
    s = splits if splits is not None else ext.gemm_fp8_splits(w.N, w.K, T)
    ws = cnt = None
    if s > 1:
        ws, cnt = workspace(x.device).ensure(ext.gemm_fp8_workspace(w.N, T, s), ext.gemm_fp8_counters(w.N, T))
    if err is None:
        err = workspace(x.device).err
    ext.gemm_fp8(w.data, w.scales, w.row_bytes, w.N, w.K, xq, xs, out, mode, s, ws, cnt, err)
    count_launch()
    return out


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


def linear_grouped(x: torch.Tensor, ws: list, out: torch.Tensor, row_counts: torch.Tensor, rows: int,
                   err: torch.Tensor | None = None) -> torch.Tensor:
    """One tcgen05 launch over up to 8 weights of one shape (routed experts): group g computes
    out[g*rows : g*rows + row_counts[g]] = x[same rows] @ W_g^T (row_counts on the device;
    token tiles past a group's count exit at once)."""
    if not ws:
        return out
    w0 = ws[0]
    if any(w.fmt != w0.fmt or w.N != w0.N or w.K != w0.K or w.row_bytes != w0.row_bytes for w in ws):
        raise ValueError("grouped GEMM: weights must share format and shape")
    if err is None:
        err = workspace(x.device).err
    require_ext().gemm_q_grouped(w0.fmt, [w.data for w in ws], [w.scales for w in ws], w0.row_bytes, w0.N, w0.K,
                                 x, rows, out, row_counts, err)
    count_launch()
    return out
