"""GGUF writer (used for checkpoints, tests and random-init benchmark models)."""
from __future__ import annotations

import os
import struct
from typing import Any

import numpy as np
import torch

from .constants import (GGUF_MAGIC, GGUF_VERSION, GGUF_DEFAULT_ALIGNMENT, GGUFValueType,
                        GGMLType, tensor_nbytes)


def _pack_str(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _infer_type(v: Any) -> GGUFValueType:
    if isinstance(v, bool):
        return GGUFValueType.BOOL
    if isinstance(v, int):
        return GGUFValueType.UINT32 if 0 <= v < 2**32 else GGUFValueType.INT64
    if isinstance(v, float):
        return GGUFValueType.FLOAT32
    if isinstance(v, str):
        return GGUFValueType.STRING
    if isinstance(v, (list, tuple)):
        return GGUFValueType.ARRAY
    raise TypeError(f"cannot encode metadata value {v!r}")


_FMT = {
    GGUFValueType.UINT8: "<B", GGUFValueType.INT8: "<b", GGUFValueType.UINT16: "<H",
    GGUFValueType.INT16: "<h", GGUFValueType.UINT32: "<I", GGUFValueType.INT32: "<i",
    GGUFValueType.FLOAT32: "<f", GGUFValueType.BOOL: "<?", GGUFValueType.UINT64: "<Q",
    GGUFValueType.INT64: "<q", GGUFValueType.FLOAT64: "<d",
}


def _pack_value(v: Any, vt: GGUFValueType | None = None) -> bytes:
    vt = vt if vt is not None else _infer_type(v)
    if vt == GGUFValueType.STRING:
        return _pack_str(v)
    if vt == GGUFValueType.ARRAY:
        items = list(v)
        if not items:
            et = GGUFValueType.INT32
        elif all(isinstance(x, str) for x in items):
            et = GGUFValueType.STRING
        elif all(isinstance(x, float) for x in items):
            et = GGUFValueType.FLOAT32
        else:
            et = GGUFValueType.INT32
        out = struct.pack("<IQ", int(et), len(items))
        if et == GGUFValueType.STRING:
            return out + b"".join(_pack_str(x) for x in items)
        arr = np.asarray(items, dtype=np.float32 if et == GGUFValueType.FLOAT32 else np.int32)
        return out + arr.astype(arr.dtype.newbyteorder("<")).tobytes()
    return struct.pack(_FMT[vt], v)


class GGUFWriter:
    """Collects metadata and tensors, then writes one GGUF v3 file.

    Tensors are given as ``uint8`` raw block tensors (already quantised) together with
    their logical row-major shape; dims are stored in ggml (innermost-first) order.
    """

    def __init__(self, path: str | os.PathLike, arch: str = "llama",
                 alignment: int = GGUF_DEFAULT_ALIGNMENT):
        self.path = os.fspath(path)
        self.alignment = alignment
        self.kv: list[tuple[str, Any, GGUFValueType | None]] = []
        self.tensors: list[tuple[str, tuple[int, ...], GGMLType, torch.Tensor]] = []
        self.add("general.architecture", arch)
        if alignment != GGUF_DEFAULT_ALIGNMENT:
            self.add("general.alignment", alignment, GGUFValueType.UINT32)

    def add(self, key: str, value: Any, vtype: GGUFValueType | None = None):
        self.kv.append((key, value, vtype))

    def add_tensor(self, name: str, raw: torch.Tensor, shape: tuple[int, ...], qtype: GGMLType):
        n = 1
        for s in shape:
            n *= s
        nb = tensor_nbytes(qtype, n)
        raw = raw.detach().to("cpu").contiguous().view(torch.uint8).reshape(-1)
        if raw.numel() != nb:
            raise ValueError(f"{name}: {raw.numel()} bytes given, {nb} expected for {GGMLType(qtype).name}{shape}")
        self.tensors.append((name, tuple(shape), GGMLType(qtype), raw))

    def write(self):
        head = bytearray()
        head += struct.pack("<IIQQ", GGUF_MAGIC, GGUF_VERSION, len(self.tensors), len(self.kv))
        for k, v, vt in self.kv:
            vt = vt if vt is not None else _infer_type(v)
            head += _pack_str(k) + struct.pack("<I", int(vt)) + _pack_value(v, vt)
        offsets = []
        off = 0
        for name, shape, qt, raw in self.tensors:
            off = (off + self.alignment - 1) // self.alignment * self.alignment
            offsets.append(off)
            off += raw.numel()
        for (name, shape, qt, raw), o in zip(self.tensors, offsets):
            dims = tuple(reversed(shape))
            head += _pack_str(name) + struct.pack("<I", len(dims))
            head += b"".join(struct.pack("<Q", d) for d in dims)
            head += struct.pack("<IQ", int(qt), o)
        pad = (-len(head)) % self.alignment
        head += b"\0" * pad
        with open(self.path, "wb") as f:
            f.write(head)
            pos = 0
            for (name, shape, qt, raw), o in zip(self.tensors, offsets):
                if o > pos:
                    f.write(b"\0" * (o - pos))
                    pos = o
                f.write(raw.numpy().tobytes())
                pos += raw.numel()
        return self.path
