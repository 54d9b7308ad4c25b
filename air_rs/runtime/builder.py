"""Constructors that wire weights, KV pool, runner and engine together."""
from __future__ import annotations

import torch

from ..gguf import GGMLType, read_gguf
from ..models.config import ModelConfig, PRESETS
from ..models.llama import LlamaWeights
from ..models.random_init import random_tensors
from ..tokenizer import Tokenizer
from .engine import Engine
from .runner import ModelRunner

from . import vram_guard


class VramBudgetError(RuntimeError):
    pass


def kv_row_bytes(head_dim: int, kv_dtype: str = "bf16") -> int:
    """Bytes of one (token, KV head) row of the paged pool: head_dim bf16 values, or for
    ``kv_dtype="fp8"`` head_dim E4M3 codes + an f32 scale + 12 bytes of padding."""
    if kv_dtype == "bf16":
        return head_dim * 2
    if kv_dtype == "fp8":
        return head_dim + 16
    raise ValueError(f"kv_dtype must be 'bf16' or 'fp8', got {kv_dtype!r}")


def kv_bytes_per_block(cfg: ModelConfig, block_size: int, tp_size: int = 1, kv_dtype: str = "bf16") -> int:
    nkv = max(1, cfg.n_kv_heads // tp_size)
    return cfg.n_layers * 2 * nkv * block_size * kv_row_bytes(cfg.head_dim, kv_dtype)


def plan_kv_blocks(cfg: ModelConfig, weights_bytes: int, *, block_size: int, device,
                   max_batch: int, max_model_len: int, tp_size: int = 1,
                   kv_fraction: float | None = None, num_blocks: int | None = None,
                   kv_dtype: str = "bf16") -> int:
    """KV blocks to allocate: enough for max_batch full-length sequences, capped by the
    VRAM guard (weights + KV <= 80 % of device memory, src/vram_guard.rs:198-337)."""
    per = kv_bytes_per_block(cfg, block_size, tp_size, kv_dtype)
    want = max_batch * ((max_model_len + block_size - 1) // block_size) + 16
    if num_blocks is not None:
        want = num_blocks
    if torch.device(device).type != "cuda":
        return want
    free, total = torch.cuda.mem_get_info(torch.device(device))
    cap = int(total * (kv_fraction or vram_guard.default_fraction()))
    used = total - free
    room = cap - used
    if room <= per * 64:
        raise VramBudgetError(f"VRAM guard: weights/other use {used/2**30:.1f} GiB of the "
                              f"{cap/2**30:.1f} GiB cap; no room for the KV pool")
    return int(min(want, room // per))


def build_runner(cfg: ModelConfig, records, *, device="cuda", max_batch=64, max_model_len=4096,
                 block_size=16, num_blocks=None, tp=None, seed=0, max_seqs=None,
                 resident: bool = True, stream_slots: int = 2, kv_alloc=None,
                 layer_range: tuple[int, int] | None = None, expert_slots: int | None = None,
                 resident_layers: int = 0, kv_dtype: str = "bf16") -> ModelRunner:
    """``resident=False``: per-layer weights stay in pinned host memory and are streamed
    through ``stream_slots`` device slots each forward (S.L.I.P. streaming mode).
    ``expert_slots``: MoE experts stay in pinned host memory and at most this many are
    resident at once (expert VRAM scheduler). ``kv_dtype="fp8"``: E4M3 paged KV pool with a
    scale per (token, head) row (about 0.56x the bf16 pool's bytes)."""
    tp_size = tp.world_size if tp is not None else 1
    tp_rank = tp.rank if tp is not None else 0
    w = LlamaWeights(cfg, records, device, tp_rank=tp_rank, tp_size=tp_size,
                     layer_device=None if resident else "cpu", layer_range=layer_range,
                     expert_device="cpu" if expert_slots else None)
    per_layer = max(1, w.nbytes() - w.resident_nbytes()) // max(1, len(w.layers))
    streamed = 0 if resident else (stream_slots + resident_layers) * per_layer
    if expert_slots:
        l0 = w.layers[0]
        streamed += expert_slots * (l0.experts_gu[0].nbytes + l0.experts_down[0].nbytes)
    nb = plan_kv_blocks(cfg, w.resident_nbytes() + streamed, block_size=block_size, device=device,
                        max_batch=max_batch, max_model_len=max_model_len, tp_size=tp_size, num_blocks=num_blocks,
                        kv_dtype=kv_dtype)
    rn = ModelRunner(cfg, w, num_blocks=nb, block_size=block_size, max_batch=max_batch,
                     max_model_len=max_model_len, device=device, tp=tp, seed=seed,
                     max_seqs=max_seqs or max(2 * max_batch + 1, 64), kv_alloc=kv_alloc, kv_dtype=kv_dtype)
    if not resident:
        rn.enable_streaming(stream_slots, resident_layers)
    if expert_slots:
        rn.enable_expert_cache(expert_slots)
    return rn


def random_engine(preset: str | ModelConfig = "tiny", qtype: GGMLType = GGMLType.Q4_K, *, seed=0,
                  device="cuda", max_batch=64, max_model_len=4096, tp=None, num_blocks=None,
                  expert_slots: int | None = None, kv_dtype: str = "bf16", **kw) -> Engine:
    """Random-init model of a named architecture built directly in HBM (no file)."""
    cfg = PRESETS[preset]() if isinstance(preset, str) else preset
    recs = random_tensors(cfg, qtype, seed=seed, device=device)
    runner = build_runner(cfg, recs, device=device, max_batch=max_batch, max_model_len=max_model_len,
                          tp=tp, num_blocks=num_blocks, seed=seed, expert_slots=expert_slots, kv_dtype=kv_dtype)
    tok = Tokenizer.byte_vocab(cfg.vocab_size, cfg.bos_token_id, cfg.eos_token_id)
    return Engine(cfg, runner, tok, max_batch=max_batch, **kw)


def engine_from_gguf(path: str, *, device=None, max_batch=64, max_model_len=None, tp=None,
                     num_blocks=None, seed=0, resident: bool | str = True, expert_slots: int | None = None,
                     parallel_read: bool = False, gds: bool = False, kv_dtype: str = "bf16", **kw) -> Engine:
    """``resident="auto"``: keep everything in HBM when it fits under the VRAM cap, else
    stream layers or serve MoE experts from host memory (``runtime.residency.plan_model``)."""
    g = read_gguf(path)
    cfg = ModelConfig.from_gguf_metadata(g.metadata).detect_layout(g.tensors)
    tok = Tokenizer.from_gguf_metadata(g.metadata)
    if device is None:
        device = "cuda" if torch.cuda.is_available() else "cpu"
    if torch.device(device).type != "cuda":
        from ..models.reference import OracleModel
        return Engine(cfg, None, tok, oracle=OracleModel.from_gguf(g), **kw)
    mml = max_model_len or min(cfg.context_length, 8192)
    stream_slots, resident_layers = 2, 0
    if resident == "auto":
        # residency plan from the device size and the checkpoint's main weight format
        from .residency import plan_model
        qt = next((t.qtype for n, t in g.tensors.items() if n.endswith("attn_q.weight")), GGMLType.Q4_K)
        total_mb = torch.cuda.get_device_properties(torch.device(device)).total_memory / 2**20
        plan = plan_model(cfg, qt, total_mb)
        resident, stream_slots = plan.resident, plan.stream_slots
        expert_slots = expert_slots or plan.expert_slots
        resident_layers = plan.resident_layers
    bufs = None
    if gds and resident is True:
        # GPUDirect Storage: file -> HBM without a host copy; threaded pread when unavailable
        try:
            bufs = g.read_gds(device)
        except OSError:
            bufs = None
    if bufs is None and (parallel_read or gds):
        bufs = g.read_parallel()
    if bufs is not None:
        recs = ((n, bufs[n], t.qtype, t.torch_shape) for n, t in g.tensors.items())
    else:
        recs = ((n, g.raw(n), t.qtype, t.torch_shape) for n, t in g.tensors.items())
    runner = build_runner(cfg, recs, device=device, max_batch=max_batch, max_model_len=mml, tp=tp,
                          num_blocks=num_blocks, seed=seed, resident=resident, expert_slots=expert_slots,
                          stream_slots=stream_slots, resident_layers=resident_layers, kv_dtype=kv_dtype)
    return Engine(cfg, runner, tok, max_batch=max_batch, **kw)


def engine_from_hf(path: str, *, qtype=GGMLType.Q4_K, device=None, max_batch=64, max_model_len=None, tp=None,
                   num_blocks=None, seed=0, tokenizer=None, kv_dtype: str = "bf16", **kw) -> Engine:
    """Engine from a Hugging Face checkpoint directory (``config.json`` + safetensors or
    ``.bin``), quantised on load to ``qtype`` (on the GPU when there is one)."""
    import json
    import os
    from ..checkpoint.hf import hf_config, hf_records
    d = path if os.path.isdir(path) else os.path.dirname(path)
    cfg = hf_config(json.load(open(os.path.join(d, "config.json"))))
    if device is None:
        device = "cuda" if torch.cuda.is_available() else "cpu"
    tok = tokenizer or Tokenizer.byte_vocab(cfg.vocab_size, cfg.bos_token_id, cfg.eos_token_id)
    recs = hf_records(path, qtype, device=device, cfg=cfg)
    if torch.device(device).type != "cuda":
        from ..models.reference import OracleModel
        t = {n: (r.cpu(), q, s) for n, r, q, s in recs}
        return Engine(cfg, None, tok, oracle=OracleModel(cfg, t), **kw)
    mml = max_model_len or min(cfg.context_length, 8192)
    runner = build_runner(cfg, recs, device=device, max_batch=max_batch, max_model_len=mml, tp=tp,
                          num_blocks=num_blocks, seed=seed, kv_dtype=kv_dtype)
    return Engine(cfg, runner, tok, max_batch=max_batch, **kw)
