"""Safetensors reader / writer (reference ``src/loader.rs:361-404`` SafetensorsLoader and
``src/strix/safetensors.rs``).

Format: an 8-byte little-endian header length N, N bytes of JSON mapping each tensor name to
``{"dtype", "shape", "data_offsets": [begin, end]}`` (offsets relative to the end of the
header; an optional ``"__metadata__"`` string map), then the raw little-endian tensor bytes.
The reader memory-maps the file, so a tensor is materialised only when asked for.
"""
from __future__ import annotations

import json
import mmap
import os
import struct

import numpy as np
import torch

_DTYPES = {"F64": torch.float64, "F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16,
           "I64": torch.int64, "I32": torch.int32, "I16": torch.int16, "I8": torch.int8, "U8": torch.uint8,
           "BOOL": torch.bool, "F8_E4M3": torch.float8_e4m3fn, "F8_E5M2": torch.float8_e5m2}
_NAMES = {v: k for k, v in _DTYPES.items()}
MAX_HEADER = 100 << 20


class SafetensorsError(ValueError):
    pass


class SafetensorsFile:
    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "rb")
        size = os.fstat(self._f.fileno()).st_size
        if size < 8:
            raise SafetensorsError(f"{path}: too short for a safetensors file")
        (n,) = struct.unpack("<Q", self._f.read(8))
        if n > MAX_HEADER or 8 + n > size:
            raise SafetensorsError(f"{path}: header length {n} out of range")
        try:
            hdr = json.loads(self._f.read(n))
        except json.JSONDecodeError as e:
            raise SafetensorsError(f"{path}: bad header JSON: {e}") from e
        self.metadata = hdr.pop("__metadata__", {}) or {}
        self._base = 8 + n
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ) if size > self._base else None
        self.tensors = {}
        for name, t in hdr.items():
            if t["dtype"] not in _DTYPES:
                raise SafetensorsError(f"{name}: unsupported dtype {t['dtype']}")
            b, e = t["data_offsets"]
            dt = _DTYPES[t["dtype"]]
            numel = 1
            for s in t["shape"]:
                numel *= s
            if e - b != numel * torch.empty((), dtype=dt).element_size() or self._base + e > size or b > e:
                raise SafetensorsError(f"{name}: data offsets {b}..{e} do not match shape {t['shape']}")
            self.tensors[name] = (dt, tuple(t["shape"]), b, e)

    def keys(self):
        return list(self.tensors)

    def get(self, name: str) -> torch.Tensor:
        dt, shape, b, e = self.tensors[name]
        if e == b:
            return torch.empty(shape, dtype=dt)
        buf = np.frombuffer(self._mm, dtype=np.uint8, count=e - b, offset=self._base + b)
        return torch.from_numpy(buf.copy()).view(dt).reshape(shape)

    def close(self):
        if self._mm is not None:
            self._mm.close()
        self._f.close()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


def load_safetensors(path: str) -> dict[str, torch.Tensor]:
    with SafetensorsFile(path) as f:
        return {k: f.get(k) for k in f.keys()}


def save_safetensors(tensors: dict[str, torch.Tensor], path: str, metadata: dict[str, str] | None = None):
    hdr, off, blobs = {}, 0, []
    for name in sorted(tensors):
        t = tensors[name].detach().contiguous().cpu()
        if t.dtype not in _NAMES:
            raise SafetensorsError(f"{name}: dtype {t.dtype} has no safetensors name")
        raw = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
        hdr[name] = {"dtype": _NAMES[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    if metadata:
        hdr["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    h = json.dumps(hdr, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)          # keep the data 8-byte aligned
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)
