"""Random-init GGUF models of named architectures (benchmarks, tests).

Weights are N(0, std) drawn from a seeded torch generator in a fixed tensor order and
quantised to the requested GGUF type; norm weights are 1.0 (F32). The same generator
and order run on CPU (to write a GGUF file) or on the GPU (to build a model in HBM
without a file), so both routes give the same quantised blocks for a given device.
"""
from __future__ import annotations

from typing import Iterator

import torch

from ..gguf import GGMLType, GGUFWriter, quantize, BLOCK_GEOMETRY
from ..tokenizer import Tokenizer
from .config import ModelConfig, FfnType


def tensor_specs(cfg: ModelConfig, qtype: GGMLType) -> Iterator[tuple[str, tuple[int, ...], GGMLType, bool]]:
    """(name, row-major shape, type, kind) in canonical order; kind is False for weights,
    True for norm weights (ones) and "bias" for biases (small random)."""
    H, V = cfg.hidden_dim, cfg.vocab_size
    yield "token_embd.weight", (V, H), qtype, False
    F = cfg.intermediate_dim
    for i in range(cfg.n_layers):
        p = f"blk.{i}."
        yield p + "attn_norm.weight", (H,), GGMLType.F32, True
        if cfg.norm_bias:
            yield p + "attn_norm.bias", (H,), GGMLType.F32, "bias"
        if cfg.fused_qkv:
            yield p + "attn_qkv.weight", (cfg.q_dim + 2 * cfg.kv_dim, H), qtype, False
        else:
            yield p + "attn_q.weight", (cfg.q_dim, H), qtype, False
            yield p + "attn_k.weight", (cfg.kv_dim, H), qtype, False
            yield p + "attn_v.weight", (cfg.kv_dim, H), qtype, False
        if cfg.qkv_bias:
            yield p + "attn_q.bias", (cfg.q_dim,), GGMLType.F32, "bias"
            yield p + "attn_k.bias", (cfg.kv_dim,), GGMLType.F32, "bias"
            yield p + "attn_v.bias", (cfg.kv_dim,), GGMLType.F32, "bias"
        yield p + "attn_output.weight", (H, cfg.q_dim), qtype, False
        yield p + "ffn_norm.weight", (H,), GGMLType.F32, True
        if cfg.norm_bias:
            yield p + "ffn_norm.bias", (H,), GGMLType.F32, "bias"
        if cfg.n_experts > 0:
            E = cfg.n_experts
            yield p + "ffn_gate_inp.weight", (E, H), GGMLType.F32, False
            yield p + "ffn_gate_exps.weight", (E, F, H), qtype, False
            yield p + "ffn_up_exps.weight", (E, F, H), qtype, False
            yield p + "ffn_down_exps.weight", (E, H, F), qtype, False
        elif cfg.ffn_type == FfnType.DENSE:
            yield p + "ffn_up.weight", (F, H), qtype, False
            yield p + "ffn_down.weight", (H, F), qtype, False
        elif cfg.fused_gate_up:
            yield p + "ffn_up.weight", (2 * F, H), qtype, False
            yield p + "ffn_down.weight", (H, F), qtype, False
        else:
            yield p + "ffn_gate.weight", (F, H), qtype, False
            yield p + "ffn_up.weight", (F, H), qtype, False
            yield p + "ffn_down.weight", (H, F), qtype, False
    yield "output_norm.weight", (H,), GGMLType.F32, True
    if cfg.norm_bias:
        yield "output_norm.bias", (H,), GGMLType.F32, "bias"
    yield "output.weight", (V, H), qtype, False


def _gen_quantised(shape, qtype, gen, std, device, chunk_rows=8192) -> torch.Tensor:
    rows = 1
    for s in shape[:-1]:
        rows *= s
    K = shape[-1]
    per, nb = BLOCK_GEOMETRY[qtype]
    out = torch.empty(rows, K // per * nb, dtype=torch.uint8, device=device)
    for r0 in range(0, rows, chunk_rows):
        r1 = min(rows, r0 + chunk_rows)
        x = torch.randn(r1 - r0, K, generator=gen, device=device, dtype=torch.float32) * std
        out[r0:r1] = quantize(x, qtype)
    return out


def random_tensors(cfg: ModelConfig, qtype: GGMLType = GGMLType.Q8_0, seed: int = 0,
                   std: float = 0.02, device: str | torch.device = "cpu"):
    """Yields (name, raw uint8 [rows, row_bytes], qtype, shape)."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    for name, shape, qt, is_norm in tensor_specs(cfg, GGMLType(qtype)):
        if is_norm == "bias":
            x = torch.randn(shape, generator=gen, device=device) * std
            raw = x.contiguous().view(torch.uint8).reshape(1, -1)
        elif is_norm:
            raw = torch.ones(shape, dtype=torch.float32, device=device).view(torch.uint8).reshape(1, -1)
        elif qt == GGMLType.F32:
            x = torch.randn(shape, generator=gen, device=device) * std
            raw = x.reshape(-1, shape[-1]).contiguous().view(torch.uint8)
        else:
            per, _ = BLOCK_GEOMETRY[qt]
            if shape[-1] % per:
                # row length not a whole number of blocks: store F16 (llama.cpp's fallback)
                qt = GGMLType.F16
            raw = _gen_quantised(shape, qt, gen, std, device)
        yield name, raw, qt, shape


def write_random_gguf(path: str, cfg: ModelConfig, qtype: GGMLType = GGMLType.Q8_0, seed: int = 0,
                      std: float = 0.02, tokenizer: Tokenizer | None = None) -> str:
    w = GGUFWriter(path, arch=cfg.arch)
    for k, v in cfg.gguf_metadata().items():
        w.add(k, v)
    tok = tokenizer or Tokenizer.byte_vocab(cfg.vocab_size, cfg.bos_token_id, cfg.eos_token_id)
    w.add("tokenizer.ggml.model", "gpt2" if tok.is_byte_level else "llama")
    w.add("tokenizer.ggml.tokens", tok.id_to_token)
    w.add("tokenizer.ggml.merges", [f"{a} {b}" for (a, b), _ in sorted(tok.merge_rank.items(), key=lambda kv: kv[1])])
    w.add("tokenizer.ggml.bos_token_id", tok.bos_id)
    w.add("tokenizer.ggml.eos_token_id", tok.eos_id)
    for name, raw, qt, shape in random_tensors(cfg, qtype, seed, std, "cpu"):
        w.add_tensor(name, raw, shape, qt)
    return w.write()
