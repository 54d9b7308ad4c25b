"""Hugging Face Llama / Mistral / Qwen2 / Mixtral checkpoints (``config.json`` + one or more
``*.safetensors`` files, or a PyTorch ``.bin`` state dict) as this framework's tensor records:
names mapped to the GGUF ones (``model.layers.N.self_attn.q_proj.weight`` ->
``blk.N.attn_q.weight`` ...), Mixtral experts stacked into ``ffn_*_exps``, and matrices
quantised on the way in (on the device given, chunk by chunk) to the requested GGUF type.

Block-scaled fp8 weights (E4M3 codes with a ``weight_scale_inv`` per 128 x 128 tile) are kept
as fp8 when the requested type is ``FP8_E4M3_B128`` (codes unchanged, the tile multiplier per
row block), else expanded with their scales first. Attention projections are kept in Hugging Face order: its rotary embedding rotates the two
halves of each head, which is the rotation the kernels apply, so no permutation is needed.
"""
from __future__ import annotations

import glob
import json
import os
import re

import torch

from ..gguf import BLOCK_GEOMETRY, GGMLType, quantize
from ..models.config import ModelConfig
from .safetensors import SafetensorsFile

_LAYER = {
    "input_layernorm.weight": "attn_norm.weight",
    "self_attn.q_proj.weight": "attn_q.weight",
    "self_attn.k_proj.weight": "attn_k.weight",
    "self_attn.v_proj.weight": "attn_v.weight",
    "self_attn.o_proj.weight": "attn_output.weight",
    "post_attention_layernorm.weight": "ffn_norm.weight",
    "mlp.gate_proj.weight": "ffn_gate.weight",
    "mlp.up_proj.weight": "ffn_up.weight",
    "mlp.down_proj.weight": "ffn_down.weight",
    "block_sparse_moe.gate.weight": "ffn_gate_inp.weight",
}
_GLOBAL = {"model.embed_tokens.weight": "token_embd.weight", "model.norm.weight": "output_norm.weight",
           "lm_head.weight": "output.weight"}
_EXPERT = re.compile(r"model\.layers\.(\d+)\.block_sparse_moe\.experts\.(\d+)\.(w1|w2|w3)\.weight")
_EXP_NAME = {"w1": "ffn_gate_exps.weight", "w3": "ffn_up_exps.weight", "w2": "ffn_down_exps.weight"}


def hf_config(cfg: dict) -> ModelConfig:
    """ModelConfig from a Hugging Face ``config.json`` dictionary."""
    H, nh = int(cfg["hidden_size"]), int(cfg["num_attention_heads"])
    arch = {"MistralForCausalLM": "mistral", "Qwen2ForCausalLM": "qwen2",
            "MixtralForCausalLM": "llama"}.get((cfg.get("architectures") or ["LlamaForCausalLM"])[0], "llama")
    eos = cfg.get("eos_token_id", 2)
    return ModelConfig(
        n_layers=int(cfg["num_hidden_layers"]), n_heads=nh,
        n_kv_heads=int(cfg.get("num_key_value_heads", nh)), hidden_dim=H,
        intermediate_dim=int(cfg["intermediate_size"]), vocab_size=int(cfg["vocab_size"]),
        rope_theta=float(cfg.get("rope_theta", 10000.0)),
        context_length=int(cfg.get("max_position_embeddings", 4096)),
        rms_norm_eps=float(cfg.get("rms_norm_eps", 1e-5)), head_dim=int(cfg.get("head_dim") or H // nh),
        arch=arch, sliding_window=cfg.get("sliding_window") or None,
        n_experts=int(cfg.get("num_local_experts", 0) or 0), moe_top_k=int(cfg.get("num_experts_per_tok", 0) or 0),
        eos_token_id=int(eos[0] if isinstance(eos, list) else eos), bos_token_id=int(cfg.get("bos_token_id", 1)))


def _open(path: str):
    """{name: lazily loaded tensor} over every checkpoint file of a directory (or one file)."""
    files = [path] if os.path.isfile(path) else sorted(glob.glob(os.path.join(path, "*.safetensors")))
    src = {}
    if files and files[0].endswith(".safetensors"):
        for fp in files:
            f = SafetensorsFile(fp)
            for k in f.keys():
                src[k] = (lambda f=f, k=k: f.get(k))
        return src
    bins = [path] if os.path.isfile(path) else sorted(glob.glob(os.path.join(path, "*.bin")))
    if not bins:
        raise FileNotFoundError(f"no safetensors or .bin checkpoint under {path}")
    for fp in bins:
        sd = torch.load(fp, map_location="cpu", weights_only=True)
        for k, v in sd.items():
            src[k] = (lambda v=v: v)
    return src


def _quantise(x: torch.Tensor, qtype: GGMLType, device, chunk_rows: int = 8192):
    """[..., K] float -> (raw uint8 [rows, row_bytes], stored type)."""
    shape = tuple(x.shape)
    x2 = x.reshape(-1, shape[-1])
    if qtype == GGMLType.F32:
        return x2.float().contiguous().view(torch.uint8), GGMLType.F32
    if qtype in (GGMLType.F16, GGMLType.BF16):
        dt = torch.float16 if qtype == GGMLType.F16 else torch.bfloat16
        return x2.to(dt).contiguous().view(torch.uint8), qtype
    per, nb = BLOCK_GEOMETRY[qtype]
    if shape[-1] % per:
        return x2.to(torch.float16).contiguous().view(torch.uint8), GGMLType.F16
    out = torch.empty(x2.shape[0], shape[-1] // per * nb, dtype=torch.uint8, device=device)
    for r0 in range(0, x2.shape[0], chunk_rows):
        out[r0:r0 + chunk_rows] = quantize(x2[r0:r0 + chunk_rows].to(device, torch.float32), qtype)
    return out, qtype


def hf_records(path: str, qtype: GGMLType = GGMLType.Q4_K, device="cpu", cfg: ModelConfig | None = None):
    """Yields (gguf name, raw, stored type, shape) for a Hugging Face checkpoint; norms and the
    MoE router stay F32, every other matrix is quantised to ``qtype``."""
    qtype = GGMLType(qtype)
    if cfg is None:
        cfg = hf_config(json.load(open(os.path.join(path if os.path.isdir(path) else os.path.dirname(path),
                                                      "config.json"))))
    src = _open(path)
    experts: dict[tuple[int, str], dict[int, torch.Tensor]] = {}
    for name in sorted(src, key=lambda n: (n.count("."), n)):
        m = _EXPERT.match(name)
        if m:
            li, e, w = int(m.group(1)), int(m.group(2)), m.group(3)
            experts.setdefault((li, w), {})[e] = src[name]
            slot = experts[(li, w)]
            if len(slot) == cfg.n_experts:
                x = torch.stack([slot[i]().float() for i in range(cfg.n_experts)])
                raw, qt = _quantise(x, qtype, device)
                yield f"blk.{li}.{_EXP_NAME[w]}", raw, qt, tuple(x.shape)
                del experts[(li, w)]
            continue
        if name in _GLOBAL:
            gname = _GLOBAL[name]
        else:
            mm = re.match(r"model\.layers\.(\d+)\.(.+)$", name)
            if not mm or mm.group(2) not in _LAYER:
                continue                      # rotary caches, biases of other families ...
            gname = f"blk.{mm.group(1)}.{_LAYER[mm.group(2)]}"
        x = src[name]()
        if (x.dtype == torch.float8_e4m3fn and qtype == GGMLType.FP8_E4M3_B128 and x.dim() == 2
                and x.shape[1] % 128 == 0 and name[: -len("weight")] + "weight_scale_inv" in src):
            # keep block-scaled fp8 as fp8: codes unchanged, tile multipliers per 128-row block
            from ..gguf.quants import fp8_b128_from_tiles
            raw = fp8_b128_from_tiles(x, src[name[: -len("weight")] + "weight_scale_inv"]()).to(device)
            yield gname, raw, GGMLType.FP8_E4M3_B128, tuple(x.shape)
            continue
        if x.dtype in (torch.float8_e4m3fn, torch.float8_e5m2):
            # block-scaled fp8 checkpoints store the tile multipliers beside the weight
            sname = name[: -len("weight")] + "weight_scale_inv"
            if sname in src:
                from ..quant.fp8 import block_dequantize_fp8
                x = block_dequantize_fp8(x, src[sname]())
            else:
                x = x.float()
        if gname.endswith("norm.weight") or gname.endswith("ffn_gate_inp.weight"):
            raw, qt = _quantise(x, GGMLType.F32, device)
        else:
            raw, qt = _quantise(x, qtype, device)
        yield gname, raw, qt, tuple(x.shape)      # tied heads reuse token_embd downstream
