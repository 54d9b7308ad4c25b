"""One engine configuration with ``AIR_`` environment overrides.

The reference spreads its settings over a hand-rolled CLI parser
(``src/bin/air_rs.rs:107-296``), ``StrixConfig`` (``src/strix/config.rs``), ``ArbConfig``
(``src/batching/arb.rs:57``), ``PdDisaggConfig`` (``src/pd_disagg.rs:588-609``) and
``PipelineConfig`` (``src/pipeline_parallel.rs:136``); model hyper-parameters come from GGUF
metadata (``src/model.rs:82-243``). Here every knob that shapes an engine lives in
``EngineConfig``; each field can be overridden by an environment variable named
``AIR_<FIELD>`` (upper case), e.g. ``AIR_MAX_BATCH=128`` or ``AIR_PREFIX_CACHE=1``, and
``build()`` makes the engine (from a GGUF file or, with ``preset``, random weights of a named
architecture).
"""
from __future__ import annotations

import dataclasses
import os
from dataclasses import dataclass, field

_TRUE = {"1", "true", "yes", "on"}
_FALSE = {"0", "false", "no", "off", ""}


@dataclass
class EngineConfig:
    model: str | None = None            # GGUF path
    preset: str | None = None           # random-init architecture name when no file is given
    qtype: str = "Q4_K"                 # weight format of random-init models
    device: str | None = None           # default: cuda when available, else the CPU oracle
    tp: int = 1
    pp: int = 1
    ep: bool = False                    # experts spread over the TP ranks
    block_size: int = 16                # KV block (tokens)
    kv_dtype: str = "bf16"              # paged KV pool: bf16 | fp8 (E4M3 + per-row scale)
    num_blocks: int | None = None       # KV pool size; default: what the VRAM guard allows
    max_batch: int = 64                 # concurrent decode rows (CUDA-graph buckets up to here)
    max_num_seqs: int = 256
    max_model_len: int | None = None
    prefill_chunk: int = 2048
    max_prefill_tokens: int = 8192
    cuda_graph_batch_sizes: tuple[int, ...] = (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 192, 256)
    resident: bool = True               # False: stream layers from pinned host memory
    stream_slots: int = 2
    expert_slots: int | None = None     # MoE experts in host memory, this many resident
    prefix_cache: bool = False
    kv_swap: bool = True
    vram_fraction: float = 0.80         # VRAM guard cap
    seed: int = 0
    draft_model: str | None = None
    draft_max: int = 5
    spec_tree: bool = False
    allreduce: str = "peer"             # TP all-reduce: fused peer kernel or "nccl"
    pressure_control: bool = False      # act on KV-pool pressure (evict cache, pause, preempt)
    secure_kv: bool = False             # zero KV blocks freed by finished requests
    admission: str = "fifo"             # fifo | priority | arb (harmonic length grouping)
    extra: dict = field(default_factory=dict)

    # ------------------------------------------------------------------ env
    @classmethod
    def from_env(cls, env: dict | None = None, **kw) -> "EngineConfig":
        """Defaults, then keyword arguments, then ``AIR_*`` variables (the environment wins)."""
        cfg = cls(**kw)
        cfg.apply_env(env)
        return cfg

    def apply_env(self, env: dict | None = None) -> "EngineConfig":
        env = os.environ if env is None else env
        for f in dataclasses.fields(self):
            if f.name == "extra":
                continue
            key = "AIR_" + f.name.upper()
            if key in env:
                setattr(self, f.name, _parse(env[key], f, getattr(self, f.name)))
        self.validate()
        return self

    def validate(self):
        if self.tp < 1 or self.pp < 1:
            raise ValueError("tp and pp must be >= 1")
        if self.block_size <= 0 or self.block_size & (self.block_size - 1):
            raise ValueError("block_size must be a power of two")
        if not 0.0 < self.vram_fraction <= 1.0:
            raise ValueError("vram_fraction must be in (0, 1]")
        if self.admission not in ("fifo", "priority", "arb"):
            raise ValueError("admission must be fifo, priority or arb")
        if self.kv_dtype not in ("bf16", "fp8"):
            raise ValueError("kv_dtype must be 'bf16' or 'fp8'")
        if self.allreduce not in ("peer", "nccl"):
            raise ValueError("allreduce must be 'peer' or 'nccl'")
        if self.stream_slots < 2:
            raise ValueError("layer streaming needs at least two slots")
        if self.model is None and self.preset is None:
            return
        if self.model is not None and self.preset is not None:
            raise ValueError("give either model or preset, not both")

    def to_dict(self) -> dict:
        return dataclasses.asdict(self)

    # ------------------------------------------------------------------ build
    def engine_kwargs(self) -> dict:
        return dict(max_batch=self.max_batch, prefill_chunk=self.prefill_chunk,
                    max_prefill_tokens=self.max_prefill_tokens, prefix_cache=self.prefix_cache,
                    pressure_control=self.pressure_control, secure_kv=self.secure_kv,
                    admission=self.admission,
                    kv_swap=self.kv_swap, cuda_graph_batch_sizes=tuple(self.cuda_graph_batch_sizes))

    def build(self, tp=None):
        """Make the engine this configuration describes (``tp`` is an optional ``TPGroup``)."""
        from .gguf import GGMLType
        from .runtime import vram_guard
        from .runtime.builder import engine_from_gguf, random_engine
        self.validate()
        vram_guard.set_default_fraction(self.vram_fraction)
        if self.model is not None:
            return engine_from_gguf(self.model, device=self.device, max_batch=self.max_batch,
                                    max_model_len=self.max_model_len, tp=tp, num_blocks=self.num_blocks,
                                    seed=self.seed, resident=self.resident, expert_slots=self.expert_slots,
                                    kv_dtype=self.kv_dtype,
                                    **{k: v for k, v in self.engine_kwargs().items() if k != "max_batch"})
        if self.preset is None:
            raise ValueError("EngineConfig needs a model path or a preset")
        return random_engine(self.preset, GGMLType[self.qtype], seed=self.seed,
                             device=self.device or "cuda", max_batch=self.max_batch,
                             max_model_len=self.max_model_len or 4096, tp=tp, num_blocks=self.num_blocks,
                             expert_slots=self.expert_slots, kv_dtype=self.kv_dtype,
                             **{k: v for k, v in self.engine_kwargs().items() if k != "max_batch"})


def _parse(raw: str, f: dataclasses.Field, current):
    t = f.type if isinstance(f.type, str) else getattr(f.type, "__name__", str(f.type))
    s = raw.strip()
    if "bool" in t:
        low = s.lower()
        if low in _TRUE:
            return True
        if low in _FALSE:
            return False
        raise ValueError(f"AIR_{f.name.upper()}: not a boolean: {raw!r}")
    if "None" in t and s.lower() in ("", "none", "null"):
        return None
    if t.startswith("tuple"):
        return tuple(int(x) for x in s.replace(" ", "").split(",") if x)
    if t.startswith("int"):
        return int(s)
    if t.startswith("float"):
        return float(s)
    return s
