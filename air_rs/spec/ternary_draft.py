"""Ternary self-drafter (reference ``src/tq2_drafter.rs`` TQ2GhostDrafter and the
``--ternary-cdsc`` mode): a draft model made from the target's own weights, each matrix
ternarised per row (absmean scale, trits in {-1, 0, +1}, BitNet b1.58 style), so speculative
decoding needs no separate draft checkpoint.

The ternary values are stored back in a block format the GEMV / GEMM kernels read (Q8_0 by
default: -s, 0 and +s are exact up to the block scale rounding), which keeps the drafter on the
same kernels as the target; the draft's accuracy is that of the ternary model.
"""
from __future__ import annotations

import torch

from ..gguf import BLOCK_GEOMETRY, GGMLType, dequantize, quantize
from ..quant.ternary import quantize_ternary

_MATRICES = ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down",
             "ffn_gate_exps", "ffn_up_exps", "ffn_down_exps")


def _ternarise_rows(w: torch.Tensor) -> torch.Tensor:
    t, s = quantize_ternary(w.float())
    return t.float() * s[:, None]


def ternary_records(records, qtype: GGMLType = GGMLType.Q8_0, device="cpu", chunk_rows: int = 4096):
    """Map (name, raw, qtype, shape) records: transformer matrices become their per-row
    ternary approximation stored as ``qtype``; embeddings, norms, router and head unchanged."""
    qtype = GGMLType(qtype)
    per, nb = BLOCK_GEOMETRY[qtype]
    for name, raw, qt, shape in records:
        base = name.split(".")[-2] if name.startswith("blk.") else ""
        if base not in _MATRICES or shape[-1] % per:
            yield name, raw, qt, shape
            continue
        rows = raw.shape[0] if raw.dim() == 2 else 1
        src = raw.reshape(rows, -1)
        out = torch.empty(rows, shape[-1] // per * nb, dtype=torch.uint8, device=device)
        for r0 in range(0, rows, chunk_rows):
            w = dequantize(src[r0:r0 + chunk_rows].to(device), GGMLType(qt)).reshape(-1, shape[-1])
            out[r0:r0 + chunk_rows] = quantize(_ternarise_rows(w), qtype)
        yield name, out, qtype, shape


def ternary_draft_engine(path: str, device="cuda", max_batch: int = 8, max_model_len: int | None = None,
                         qtype: GGMLType = GGMLType.Q8_0, **kw):
    """Draft engine built from a GGUF target with ternarised matrices."""
    from ..gguf import read_gguf
    from ..models.config import ModelConfig
    from ..runtime.builder import build_runner
    from ..runtime.engine import Engine
    from ..tokenizer import Tokenizer
    g = read_gguf(path)
    cfg = ModelConfig.from_gguf_metadata(g.metadata)
    tok = Tokenizer.from_gguf_metadata(g.metadata)
    recs = ternary_records(((n, g.raw(n), t.qtype, t.torch_shape) for n, t in g.tensors.items()), qtype,
                           device=device if torch.device(device).type == "cuda" else "cpu")
    if torch.device(device).type != "cuda":
        from ..models.reference import OracleModel
        return Engine(cfg, None, tok, oracle=OracleModel(cfg, {n: (r, q, s) for n, r, q, s in recs}), **kw)
    rn = build_runner(cfg, recs, device=device, max_batch=max_batch,
                      max_model_len=max_model_len or min(cfg.context_length, 8192))
    return Engine(cfg, rn, tok, max_batch=max_batch, **kw)
