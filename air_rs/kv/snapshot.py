"""KV session snapshots: a sequence's paged KV blocks plus its token ids, written to a file and
loaded back into the pool of a later engine.

The reference persists no session state: resume inside a session is
``SessionKvCache::truncate_to`` (``src/kv_cache.rs:364``) and ``*.draft.json`` sidecars are
described but never written. Here a snapshot is one file:

* header: format version, pool geometry (layers, KV heads, block size, head dim, dtype), the
  token ids whose KV is stored, and a CRC-32 of the KV bytes;
* payload: ``kv[:, blocks]`` of the sequence (``[L, n_blocks, 2, n_kv, block, d]``), gathered
  on the device and copied to the host once.

Loading checks the geometry and the checksum (a corrupt or foreign file raises
``SnapshotError`` and touches nothing), allocates fresh blocks, copies the payload into them
and, in the engine, hands the whole blocks to the prefix cache so the next request whose
prompt starts with those tokens skips their prefill.
"""
from __future__ import annotations

import io
import zlib
from dataclasses import dataclass

import torch

VERSION = 1


class SnapshotError(RuntimeError):
    pass


@dataclass
class SnapshotInfo:
    tokens: list[int]
    n_blocks: int
    block_size: int
    nbytes: int


def _geometry(kv: torch.Tensor) -> dict:
    L, _, two, nkv, bs, d = kv.shape
    return {"layers": L, "two": two, "n_kv": nkv, "block_size": bs, "head_dim": d, "dtype": str(kv.dtype)}


def _crc(t: torch.Tensor) -> int:
    return zlib.crc32(t.contiguous().view(torch.uint8).numpy().tobytes()) & 0xFFFFFFFF


def save(path, kv: torch.Tensor, blocks: list[int], tokens: list[int]) -> SnapshotInfo:
    """Write the KV of ``tokens`` (held in ``blocks``, in order) to ``path``."""
    bs = kv.shape[4]
    need = (len(tokens) + bs - 1) // bs
    if need > len(blocks):
        raise SnapshotError(f"{len(tokens)} tokens need {need} blocks, sequence holds {len(blocks)}")
    idx = torch.tensor(blocks[:need], dtype=torch.long, device=kv.device)
    host = kv.index_select(1, idx).cpu()
    payload = {"version": VERSION, "geometry": _geometry(kv), "tokens": list(map(int, tokens)),
               "crc32": _crc(host), "kv": host}
    buf = io.BytesIO()
    torch.save(payload, buf)
    with open(path, "wb") as f:
        f.write(buf.getvalue())
    return SnapshotInfo(list(tokens), need, bs, host.numel() * host.element_size())


def read(path, kv: torch.Tensor | None = None) -> dict:
    """Load and validate a snapshot (geometry against ``kv`` when given)."""
    try:
        with open(path, "rb") as f:
            payload = torch.load(io.BytesIO(f.read()), map_location="cpu", weights_only=True)
    except Exception as e:  # truncated / not a snapshot
        raise SnapshotError(f"unreadable snapshot {path}: {e}") from e
    if not isinstance(payload, dict) or payload.get("version") != VERSION:
        raise SnapshotError(f"{path}: not a version-{VERSION} KV snapshot")
    if kv is not None and payload["geometry"] != _geometry(kv):
        raise SnapshotError(f"{path}: pool geometry {payload['geometry']} does not match {_geometry(kv)}")
    if _crc(payload["kv"]) != payload["crc32"]:
        raise SnapshotError(f"{path}: KV checksum mismatch")
    return payload


def load_into(path, kv: torch.Tensor, seqs) -> tuple[int, list[int], list[int]]:
    """Allocate a new sequence holding the snapshot's KV; returns (seq id, tokens, blocks)."""
    p = read(path, kv)
    toks = p["tokens"]
    host = p["kv"]
    if not seqs.allocator.can_allocate(host.shape[1]):
        raise SnapshotError(f"pool has no room for {host.shape[1]} blocks")
    seq = seqs.create_sequence()
    seqs.append(seq, len(toks))
    blocks = list(seqs.block_table(seq))
    idx = torch.tensor(blocks, dtype=torch.long, device=kv.device)
    kv.index_copy_(1, idx, host.to(kv.device, non_blocking=False))
    return seq, toks, blocks
