"""Llama-family transformer on the sm_100a kernels (Llama / Mistral / Qwen2 shapes).

Weights live in HBM in kernel-native formats (``QWeight``); Q/K/V rows are concatenated
into one matrix and gate/up into another so each layer is five weight streams. The
decode step (batch <= 8) is

    norm+quant -> QKV GEMV (+RoPE, +paged KV write) -> paged attention (+quant)
    -> O GEMV (+residual) -> norm+quant -> gate|up GEMV (+SwiGLU) -> quant
    -> down GEMV (+residual)

which replaces the reference's per-layer candle path (``src/model.rs:460-745``) and its
host round trips of the KV cache (``src/kv_cache.rs:244-339``). Prefill and large-batch
decode go through ``linear`` (tcgen05 GEMM) with token-parallel RoPE/KV, SwiGLU and
residual kernels, and the same paged attention kernel.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Iterable

import torch

from .. import ops
from ..gguf import GGMLType
from ..gguf.quants import dequantize
from .config import ModelConfig, FfnType


@dataclass
class LayerWeights:
    attn_norm: torch.Tensor
    wqkv: ops.QWeight
    wo: ops.QWeight
    ffn_norm: torch.Tensor
    wgu: ops.QWeight | None          # [2F, H]: gate rows then up rows
    wdown: ops.QWeight | None
    # MoE
    router: torch.Tensor | None = None      # [E, H] f32
    experts_gu: list = field(default_factory=list)
    experts_down: list = field(default_factory=list)
    expert_ids: list = field(default_factory=list)   # global ids of the local experts
    # architecture variants (reference src/model.rs:326-360)
    qkv_bias: torch.Tensor | None = None    # [q|k|v] rows of this rank, f32 (Qwen2)
    attn_norm_b: torch.Tensor | None = None  # LayerNorm biases (Falcon)
    ffn_norm_b: torch.Tensor | None = None

    @property
    def w_gate(self) -> ops.QWeight:
        return self.wgu.part(0)

    @property
    def w_up(self) -> ops.QWeight:
        return self.wgu.part(1)


def layer_tensors(lw: "LayerWeights") -> list:
    """Every tensor of a layer in a fixed order (weights data/scales, norms, router)."""
    out = [lw.attn_norm, lw.ffn_norm] + [t for t in (lw.qkv_bias, lw.attn_norm_b, lw.ffn_norm_b) if t is not None]
    qws = [lw.wqkv, lw.wo] + ([lw.wgu, lw.wdown] if lw.wgu is not None else []) + list(lw.experts_gu) + \
        list(lw.experts_down)
    for q in qws:
        out.append(q.data)
        if q.scales is not None:
            out.append(q.scales)
    if lw.router is not None:
        out.append(lw.router)
    return out


def pin_layer(lw: "LayerWeights"):
    """Move a host-resident layer's tensors into page-locked memory (in place)."""
    import dataclasses
    for f in dataclasses.fields(lw):
        v = getattr(lw, f.name)
        if isinstance(v, torch.Tensor):
            setattr(lw, f.name, v.pin_memory())
        elif isinstance(v, ops.QWeight):
            setattr(lw, f.name, v.to_device(None, pin=True))
        elif isinstance(v, list) and v and isinstance(v[0], ops.QWeight):
            setattr(lw, f.name, [q.to_device(None, pin=True) for q in v])


class LlamaWeights:
    """Device-resident weights, built from (name, raw, qtype, shape) records."""

    def __init__(self, cfg: ModelConfig, records: Iterable, device, tp_rank: int = 0, tp_size: int = 1,
                 layer_device=None, layer_range: tuple[int, int] | None = None, expert_device=None):
        """``layer_device`` (default: ``device``) holds the per-layer weights; ``"cpu"`` keeps
        them in pinned host memory for layer streaming (S.L.I.P.). ``expert_device="cpu"`` keeps
        only the MoE experts in pinned host memory (served through an expert cache)."""
        self.cfg = cfg
        self.device = torch.device(device)
        self.layer_device = torch.device(layer_device) if layer_device is not None else self.device
        self.expert_device = torch.device(expert_device) if expert_device is not None else None
        # pipeline stage: only layers [l0, l1) are loaded (indexed from 0 here)
        self.layer_range = tuple(layer_range) if layer_range is not None else (0, cfg.n_layers)
        self.tp_rank, self.tp_size = tp_rank, tp_size
        pending: dict[str, tuple] = {}
        self.layers: list[LayerWeights | None] = [None] * (self.layer_range[1] - self.layer_range[0])
        self.embd = self.out_norm = self.lm_head = None
        self.out_norm_b = None
        for name, raw, qt, shape in records:
            pending[name] = (raw, GGMLType(qt), tuple(shape))
            self._try_build(pending)
        if self.lm_head is None and "token_embd.weight" in pending:
            self.lm_head = self._lin_full(*pending["token_embd.weight"])
        self._try_build(pending, final=True)
        missing = [i for i, l in enumerate(self.layers) if l is None]
        if missing or self.embd is None or self.out_norm is None or self.lm_head is None:
            raise ValueError(f"incomplete checkpoint: layers {missing[:4]}... or globals missing")

    # -- helpers -------------------------------------------------------------
    def _vec(self, raw, qt, shape):
        return dequantize(raw.reshape(1, -1), qt).reshape(-1).float().to(self.device)

    def _lin_full(self, raw, qt, shape):
        return ops.QWeight.from_raw(raw, qt, shape[0], shape[1], self.device)

    def _lin_rows(self, raw, qt, shape, r0, r1):
        return ops.QWeight.from_raw(raw.reshape(shape[0], -1)[r0:r1], qt, r1 - r0, shape[1], self.device)

    def _lin_cols(self, raw, qt, shape, c0, c1):
        """Input-dim shard: whole quant blocks of each row (row-parallel TP)."""
        from ..gguf import BLOCK_GEOMETRY
        per, nb = BLOCK_GEOMETRY[qt]
        if c0 % per or c1 % per:
            raise ValueError(f"TP shard boundary {c0}:{c1} not aligned to {qt.name} block {per}")
        r = raw.reshape(shape[0], -1)[:, c0 // per * nb: c1 // per * nb]
        return ops.QWeight.from_raw(r.contiguous(), qt, shape[0], c1 - c0, self.device)

    def _try_build(self, p: dict, final: bool = False):
        cfg = self.cfg
        if self.embd is None and "token_embd.weight" in p:
            raw, qt, shape = p["token_embd.weight"]
            if qt == GGMLType.FP8_E4M3_B128:
                # the embedding gather reads GGUF block formats; keep the table as Q8_0
                from ..gguf.quants import quantize_q8_0
                raw, qt = quantize_q8_0(dequantize(raw.reshape(shape[0], -1), qt)), GGMLType.Q8_0
            self.embd = self._lin_full(raw, qt, shape)
        if self.out_norm is None and "output_norm.weight" in p:
            self.out_norm = self._vec(*p.pop("output_norm.weight"))
        if self.out_norm_b is None and "output_norm.bias" in p:
            self.out_norm_b = self._vec(*p.pop("output_norm.bias"))
        if self.lm_head is None and "output.weight" in p:
            raw, qt, shape = p.pop("output.weight")
            self.lm_head = self._shard_rows_tp(raw, qt, shape)
        l0, l1 = self.layer_range
        for i in range(cfg.n_layers):
            if not l0 <= i < l1:
                for k in [k for k in p if k.startswith(f"blk.{i}.")]:
                    del p[k]                 # another pipeline stage's layer
                continue
            if self.layers[i - l0] is not None:
                continue
            pre = f"blk.{i}."
            need = ["attn_norm.weight", "attn_output.weight", "ffn_norm.weight"]
            need += ["attn_qkv.weight"] if cfg.fused_qkv else ["attn_q.weight", "attn_k.weight", "attn_v.weight"]
            if cfg.qkv_bias:
                need += ["attn_q.bias", "attn_k.bias", "attn_v.bias"]
            if cfg.norm_bias:
                need += ["attn_norm.bias", "ffn_norm.bias"]
            if cfg.n_experts:
                need += ["ffn_gate_inp.weight", "ffn_gate_exps.weight", "ffn_up_exps.weight",
                         "ffn_down_exps.weight"]
            elif cfg.ffn_type == FfnType.DENSE or cfg.fused_gate_up:
                need += ["ffn_up.weight", "ffn_down.weight"]
            else:
                need += ["ffn_gate.weight", "ffn_up.weight", "ffn_down.weight"]
            if not all(pre + n in p for n in need):
                continue
            g = {n: p.pop(pre + n) for n in need}
            dev, self.device = self.device, self.layer_device
            try:
                self.layers[i - l0] = self._build_layer(g)
            finally:
                self.device = dev
            if self.layer_device.type == "cpu" and dev.type == "cuda":
                pin_layer(self.layers[i - l0])

    def _shard_rows_tp(self, raw, qt, shape):
        if self.tp_size == 1:
            return self._lin_full(raw, qt, shape)
        n = shape[0]
        per = (n + self.tp_size - 1) // self.tp_size
        r0, r1 = self.tp_rank * per, min(n, (self.tp_rank + 1) * per)
        return self._lin_rows(raw, qt, shape, r0, r1)

    def _build_layer(self, g) -> LayerWeights:
        cfg, tp, rk = self.cfg, self.tp_size, self.tp_rank
        hd = cfg.head_dim
        nh_l, nkv_l = cfg.n_heads // tp, max(1, cfg.n_kv_heads // tp)
        kv_rank = rk * nkv_l // max(1, nkv_l) if cfg.n_kv_heads >= tp else rk * cfg.n_kv_heads // tp
        q0, q1 = rk * nh_l * hd, (rk + 1) * nh_l * hd
        if cfg.n_kv_heads >= tp:
            k0 = rk * nkv_l * hd
        else:  # replicate KV heads across ranks that share them
            k0 = (rk * cfg.n_kv_heads // tp) * hd
        k1 = k0 + nkv_l * hd
        if cfg.fused_qkv:    # Phi-3: rows [q; k; v] of one tensor
            raw, qt, shp = g["attn_qkv.weight"]
            qd, kd = cfg.q_dim, cfg.kv_dim
            q = self._lin_rows(raw, qt, shp, q0, q1)
            k = self._lin_rows(raw, qt, shp, qd + k0, qd + k1)
            v = self._lin_rows(raw, qt, shp, qd + kd + k0, qd + kd + k1)
        else:
            q = self._lin_rows(*g["attn_q.weight"], q0, q1)
            k = self._lin_rows(*g["attn_k.weight"], k0, k1)
            v = self._lin_rows(*g["attn_v.weight"], k0, k1)
        del kv_rank
        wqkv = ops.QWeight.cat([q, k, v])
        if tp == 1:
            wo = self._lin_full(*g["attn_output.weight"])
        else:
            wo = self._lin_cols(*g["attn_output.weight"], rk * nh_l * hd, (rk + 1) * nh_l * hd)
        lw = LayerWeights(self._vec(*g["attn_norm.weight"]), wqkv, wo, self._vec(*g["ffn_norm.weight"]),
                          None, None)
        if cfg.qkv_bias:
            bq, bk, bv = (self._vec(*g[f"attn_{n}.bias"]) for n in "qkv")
            lw.qkv_bias = torch.cat([bq[q0:q1], bk[k0:k1], bv[k0:k1]]).contiguous()
        if cfg.norm_bias:
            lw.attn_norm_b, lw.ffn_norm_b = self._vec(*g["attn_norm.bias"]), self._vec(*g["ffn_norm.bias"])
        F = cfg.intermediate_dim
        Fl = F // tp
        if cfg.n_experts:
            lw.router = dequantize(g["ffn_gate_inp.weight"][0], g["ffn_gate_inp.weight"][1]).reshape(
                cfg.n_experts, cfg.hidden_dim).float().to(self.device)
            for name, dst in (("ffn_gate_exps.weight", None),):
                pass
            gr, gq, gs = g["ffn_gate_exps.weight"]
            ur, uq, us = g["ffn_up_exps.weight"]
            dr, dq, dsh = g["ffn_down_exps.weight"]
            E = cfg.n_experts
            gr = gr.reshape(E, F, -1)
            ur = ur.reshape(E, F, -1)
            dr = dr.reshape(E, cfg.hidden_dim, -1)
            # expert parallelism: under TP the experts are spread over the ranks (expert e on
            # rank e % tp); attention stays tensor parallel
            lw.expert_ids = [e for e in range(E) if e % tp == rk]
            xdev = self.expert_device or self.device
            pin = xdev.type == "cpu" and self.device.type == "cuda"
            for e in lw.expert_ids:
                ge = ops.QWeight.from_raw(gr[e], gq, F, cfg.hidden_dim, xdev)
                ue = ops.QWeight.from_raw(ur[e], uq, F, cfg.hidden_dim, xdev)
                gu = ops.QWeight.cat([ge, ue])
                dn = ops.QWeight.from_raw(dr[e], dq, cfg.hidden_dim, F, xdev)
                lw.experts_gu.append(gu.to_device(None, pin=True) if pin else gu)
                lw.experts_down.append(dn.to_device(None, pin=True) if pin else dn)
        elif cfg.ffn_type == FfnType.DENSE:
            # Falcon: up -> GELU -> down; wgu holds only the up rows (no gate)
            lw.wgu = self._lin_rows(*g["ffn_up.weight"], rk * Fl, (rk + 1) * Fl)
            if tp == 1:
                lw.wdown = self._lin_full(*g["ffn_down.weight"])
            else:
                lw.wdown = self._lin_cols(*g["ffn_down.weight"], rk * Fl, (rk + 1) * Fl)
        else:
            if cfg.fused_gate_up:   # Phi-3: ffn_up = [gate; up]
                raw, qt, shp = g["ffn_up.weight"]
                gate = self._lin_rows(raw, qt, shp, rk * Fl, (rk + 1) * Fl)
                up = self._lin_rows(raw, qt, shp, F + rk * Fl, F + (rk + 1) * Fl)
            else:
                gate = self._lin_rows(*g["ffn_gate.weight"], rk * Fl, (rk + 1) * Fl)
                up = self._lin_rows(*g["ffn_up.weight"], rk * Fl, (rk + 1) * Fl)
            lw.wgu = ops.QWeight.cat([gate, up])
            if tp == 1:
                lw.wdown = self._lin_full(*g["ffn_down.weight"])
            else:
                lw.wdown = self._lin_cols(*g["ffn_down.weight"], rk * Fl, (rk + 1) * Fl)
        return lw

    def resident_nbytes(self) -> int:
        """Bytes on the compute device (layers streamed from host memory excluded)."""
        if self.layer_device == self.device:
            n = self.nbytes()
            if self.expert_device is not None and self.expert_device != self.device:
                n -= sum(e.nbytes for l in self.layers for e in l.experts_gu + l.experts_down)
            return n
        return self.embd.nbytes + self.lm_head.nbytes

    def nbytes(self) -> int:
        n = self.embd.nbytes + self.lm_head.nbytes
        for l in self.layers:
            n += l.wqkv.nbytes + l.wo.nbytes
            if l.wgu is not None:
                n += l.wgu.nbytes + l.wdown.nbytes
            for e in l.experts_gu + l.experts_down:
                n += e.nbytes
        return n
