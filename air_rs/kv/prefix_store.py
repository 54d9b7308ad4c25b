"""Per-model prefix KV store with a compression tag per entry (reference ``src/prefix_kv.rs``:
CompressionScheme {F16, Bf16, Q8, OneBit}, PrefixEntry, PrefixKvCache with store / restore /
contains / entry_scheme / prefix_len / entry_size_bytes / evict / evict_all / summary and
FIFO eviction).

A serving node that hosts several models (``air_rs.sched.mux``) keeps, per model id, the KV
of that model's fixed system prompt in host memory, so a new request for the model restores
it into the device pool instead of prefilling it. The entry holds whole paged-KV blocks
[L, n, 2, n_kv, bs, d] taken straight from the pool; ``scheme`` decides how they are kept:

* ``BF16`` / ``F16``: bit-exact copies (F16 converts from the pool's dtype);
* ``Q8``: int8 with one scale per 32 values (``quant.int8.kv_q8_0_encode``) — 8.5 bits;
* ``ONEBIT``: keys as mean-centred sign bits with a norm and mean per row, values as 8-bit
  affine codes (``kv.compress``) — for warm tiers where an approximate prefix is acceptable.

``restore`` allocates a sequence in the ``SequenceManager`` and writes the decoded blocks
into the pool; with a prefix cache attached the caller inserts the full blocks there.
"""
from __future__ import annotations

import enum
import time
from collections import OrderedDict
from dataclasses import dataclass, field

import torch

from ..quant.int8 import kv_q8_0_decode, kv_q8_0_encode
from .compress import CompressedKeys, CompressedValues


class CompressionScheme(str, enum.Enum):
    F16 = "f16"
    BF16 = "bf16"
    Q8 = "q8"
    ONEBIT = "1bit"

    def compression_ratio(self) -> float:
        """Size of a 16-bit cache over the size of this encoding (d = 128)."""
        return {CompressionScheme.F16: 1.0, CompressionScheme.BF16: 1.0,
                CompressionScheme.Q8: 16 / 8.5,
                CompressionScheme.ONEBIT: 2 * 16 / (1 + 8 * 8 / 128 + 8 + 8 * 8 / 128)}[self]

    def label(self) -> str:
        return {CompressionScheme.F16: "F16 (raw)", CompressionScheme.BF16: "BF16 (raw)",
                CompressionScheme.Q8: "Q8 (int8, 32-value groups)",
                CompressionScheme.ONEBIT: "1-bit keys + 8-bit values"}[self]

    def lossless(self) -> bool:
        return self in (CompressionScheme.BF16,)


@dataclass
class PrefixEntry:
    model_id: str
    tokens: list[int]
    scheme: CompressionScheme
    shape: tuple                   # [L, n_blocks, 2, n_kv, bs, d] of the blocks kept
    dtype: torch.dtype             # the pool's dtype
    payload: dict
    created: float = field(default_factory=time.time)

    def size_bytes(self) -> int:
        n = 0
        for v in self.payload.values():
            if isinstance(v, torch.Tensor):
                n += v.numel() * v.element_size()
        return n

    def n_blocks(self) -> int:
        return self.shape[1]


def _encode(blocks: torch.Tensor, scheme: CompressionScheme) -> dict:
    if blocks.dtype == torch.uint8:
        # fp8 pool rows (E4M3 codes + scale) are already compressed: kept byte for byte
        return {"kv": blocks.clone()}
    if scheme == CompressionScheme.BF16:
        return {"kv": blocks.to(torch.bfloat16).clone()}
    if scheme == CompressionScheme.F16:
        return {"kv": blocks.to(torch.float16).clone()}
    if scheme == CompressionScheme.Q8:
        q, s = kv_q8_0_encode(blocks)
        return {"q": q, "s": s}
    d = blocks.shape[-1]
    k = blocks[:, :, 0].reshape(-1, d)
    v = blocks[:, :, 1].reshape(-1, d)
    ck, cv = CompressedKeys.compress(k), CompressedValues.compress(v)
    return {"k_sign": ck.sign_bits, "k_mag": ck.magnitude, "k_mean": ck.mean,
            "v_data": cv.data, "v_scale": cv.scale, "v_min": cv.min_val}


def _decode(e: PrefixEntry) -> torch.Tensor:
    p, shape = e.payload, e.shape
    if e.scheme in (CompressionScheme.BF16, CompressionScheme.F16):
        return p["kv"].to(e.dtype)
    if e.scheme == CompressionScheme.Q8:
        return kv_q8_0_decode(p["q"], p["s"]).to(e.dtype)
    d = shape[-1]
    k = CompressedKeys(p["k_sign"], p["k_mag"], p["k_mean"], d).decompress()
    v = CompressedValues(p["v_data"], p["v_scale"], p["v_min"]).decompress()
    half = (shape[0], shape[1], *shape[3:])
    return torch.stack([k.reshape(half), v.reshape(half)], 2).to(e.dtype)


class PrefixKvStore:
    """model id -> PrefixEntry, at most ``max_entries`` (oldest stored evicted first) and, when
    given, at most ``max_bytes`` in total."""

    def __init__(self, max_entries: int = 4, max_bytes: int | None = None):
        if max_entries < 1:
            raise ValueError("max_entries must be >= 1")
        self.max_entries, self.max_bytes = max_entries, max_bytes
        self._e: "OrderedDict[str, PrefixEntry]" = OrderedDict()
        self.hits = self.misses = self.evictions = 0

    # ---------------------------------------------------------------- store / restore
    def store(self, model_id: str, kv: torch.Tensor, blocks: list[int], tokens: list[int],
              scheme: CompressionScheme | str = CompressionScheme.BF16) -> PrefixEntry:
        """Keep the KV of ``tokens`` (held in pool blocks ``blocks``, in order), replacing
        any entry of the model."""
        scheme = CompressionScheme(scheme)
        bs = kv.shape[4]
        need = (len(tokens) + bs - 1) // bs
        if not tokens or need > len(blocks):
            raise ValueError(f"{len(tokens)} tokens need {need} blocks, {len(blocks)} given")
        if kv.dtype == torch.uint8 and scheme != CompressionScheme.BF16:
            raise ValueError("an fp8 KV pool is stored as is (scheme BF16 = raw rows)")
        if scheme == CompressionScheme.Q8 and kv.shape[-1] % 32:
            raise ValueError("Q8 needs a head dim that is a multiple of 32")
        idx = torch.tensor(blocks[:need], dtype=torch.long, device=kv.device)
        host = kv.index_select(1, idx).cpu()
        e = PrefixEntry(model_id, list(map(int, tokens)), scheme, tuple(host.shape), kv.dtype, _encode(host, scheme))
        if self.max_bytes is not None and e.size_bytes() > self.max_bytes:
            raise ValueError(f"prefix of {e.size_bytes()} bytes exceeds the store's {self.max_bytes}")
        self._e.pop(model_id, None)
        self._e[model_id] = e
        while len(self._e) > self.max_entries or (self.max_bytes is not None and self.total_bytes() > self.max_bytes):
            self._e.popitem(last=False)
            self.evictions += 1
        return e

    def restore(self, model_id: str, kv: torch.Tensor, seqs) -> tuple[int, list[int], list[int]]:
        """New sequence holding the model's prefix KV: (seq id, tokens, blocks). KeyError when
        the model has no entry; RuntimeError when the pool geometry differs or is full."""
        e = self._e.get(model_id)
        if e is None:
            self.misses += 1
            raise KeyError(f"no prefix stored for model {model_id!r}")
        want = (kv.shape[0], kv.shape[2], kv.shape[3], kv.shape[4], kv.shape[5])
        have = (e.shape[0], e.shape[2], e.shape[3], e.shape[4], e.shape[5])
        if want != have or kv.dtype != e.dtype:
            raise RuntimeError(f"prefix of {model_id!r} has geometry {have}/{e.dtype}, pool {want}/{kv.dtype}")
        if not seqs.allocator.can_allocate(e.n_blocks()):
            raise RuntimeError(f"pool has no room for {e.n_blocks()} blocks")
        data = _decode(e)
        seq = seqs.create_sequence()
        seqs.append(seq, len(e.tokens))
        blocks = list(seqs.block_table(seq))
        kv.index_copy_(1, torch.tensor(blocks, dtype=torch.long, device=kv.device), data.to(kv.device))
        self.hits += 1
        return seq, list(e.tokens), blocks

    # ---------------------------------------------------------------- queries
    def contains(self, model_id: str) -> bool:
        return model_id in self._e

    def __len__(self) -> int:
        return len(self._e)

    def is_empty(self) -> bool:
        return not self._e

    def entry_scheme(self, model_id: str) -> CompressionScheme | None:
        e = self._e.get(model_id)
        return None if e is None else e.scheme

    def prefix_len(self, model_id: str) -> int | None:
        e = self._e.get(model_id)
        return None if e is None else len(e.tokens)

    def entry_size_bytes(self, model_id: str) -> int | None:
        e = self._e.get(model_id)
        return None if e is None else e.size_bytes()

    def total_bytes(self) -> int:
        return sum(e.size_bytes() for e in self._e.values())

    def evict(self, model_id: str) -> bool:
        return self._e.pop(model_id, None) is not None

    def evict_all(self):
        self._e.clear()

    def summary(self) -> str:
        rows = [f"{m}: {len(e.tokens)} tokens, {e.scheme.label()}, {e.size_bytes() / 2**20:.2f} MiB"
                for m, e in self._e.items()]
        return (f"prefix store: {len(self._e)}/{self.max_entries} models, {self.total_bytes() / 2**20:.2f} MiB, "
                f"hits {self.hits}, misses {self.misses}, evictions {self.evictions}"
                + "".join("\n  " + r for r in rows))
