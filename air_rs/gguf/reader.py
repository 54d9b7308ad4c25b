"""Memory-mapped GGUF reader.

Parses the header (metadata key/values and the tensor index) and exposes every tensor as
a zero-copy ``uint8`` view of the mapped file. Mirrors what the reference's loader and
streamer read (``src/loader.rs:70-357``, ``src/weight_streamer.rs:57-139``): absolute data
offsets (``TensorRecord``), the ``general.alignment`` rule, and the tokenizer arrays.
"""
from __future__ import annotations

import mmap
import os
import struct
import warnings
from dataclasses import dataclass, field
from typing import Any

import numpy as np
import torch

from .constants import (GGUF_MAGIC, GGUF_DEFAULT_ALIGNMENT, GGUFValueType, GGMLType,
                        tensor_nbytes)

_SCALAR = {
    GGUFValueType.UINT8: "<B", GGUFValueType.INT8: "<b",
    GGUFValueType.UINT16: "<H", GGUFValueType.INT16: "<h",
    GGUFValueType.UINT32: "<I", GGUFValueType.INT32: "<i",
    GGUFValueType.FLOAT32: "<f", GGUFValueType.BOOL: "<?",
    GGUFValueType.UINT64: "<Q", GGUFValueType.INT64: "<q",
    GGUFValueType.FLOAT64: "<d",
}
_NP = {
    GGUFValueType.UINT8: np.uint8, GGUFValueType.INT8: np.int8,
    GGUFValueType.UINT16: np.uint16, GGUFValueType.INT16: np.int16,
    GGUFValueType.UINT32: np.uint32, GGUFValueType.INT32: np.int32,
    GGUFValueType.FLOAT32: np.float32, GGUFValueType.BOOL: np.bool_,
    GGUFValueType.UINT64: np.uint64, GGUFValueType.INT64: np.int64,
    GGUFValueType.FLOAT64: np.float64,
}


class GGUFError(ValueError):
    pass


@dataclass
class TensorInfo:
    name: str
    shape: tuple[int, ...]      # ggml order: shape[0] is the innermost (row length)
    qtype: GGMLType
    offset: int                 # absolute byte offset in the file
    nbytes: int

    @property
    def n_elements(self) -> int:
        n = 1
        for s in self.shape:
            n *= s
        return n

    @property
    def rows(self) -> int:
        return self.n_elements // self.shape[0]

    @property
    def torch_shape(self) -> tuple[int, ...]:
        """Row-major (PyTorch) logical shape: reversed ggml dims."""
        return tuple(reversed(self.shape))


@dataclass
class GGUFFile:
    path: str
    version: int
    metadata: dict[str, Any]
    tensors: dict[str, TensorInfo]
    alignment: int
    data_offset: int
    _mm: Any = field(default=None, repr=False)
    _buf: Any = field(default=None, repr=False)

    # -- tensor access -----------------------------------------------------
    def raw(self, name: str) -> torch.Tensor:
        """Zero-copy uint8 view ``[rows, row_bytes]`` of a tensor's blocks."""
        t = self.tensors[name]
        flat = self._buf[t.offset:t.offset + t.nbytes]
        return flat.view(t.rows, t.nbytes // t.rows)

    def read_parallel(self, names=None, workers: int = 8, pin: bool | None = None) -> dict:
        """Tensors read with ``workers`` threads of ``pread`` into (pinned) host buffers
        instead of page faults on the memory map: globals first, then layer by layer, so a
        cold start from NVMe keeps several requests in flight. Returns name -> uint8
        ``[rows, row_bytes]`` like ``raw``."""
        from ..stream.strix import IoEngine, IoPriority, IoRequest
        names = list(self.tensors) if names is None else list(names)

        def order(n):
            if n.startswith("blk."):
                return (1, int(n.split(".")[1]))
            return (0, 0)
        eng = IoEngine(self.path, capacity=workers, workers=workers, pin=pin)
        try:
            for n in sorted(names, key=order):
                t = self.tensors[n]
                pr = IoPriority.CRITICAL if not n.startswith("blk.") else IoPriority.NORMAL
                eng.submit(IoRequest(n, t.offset, t.nbytes, pr))
            done = eng.wait_all(timeout=3600.0)
        finally:
            eng.close()
        out = {}
        for c in done:
            if c.error:
                raise OSError(f"reading {c.tensor_id} from {self.path}: {c.error}")
            t = self.tensors[c.tensor_id]
            out[c.tensor_id] = c.data.view(t.rows, t.nbytes // t.rows)
        if len(out) != len(names):
            raise OSError(f"{len(names) - len(out)} tensors of {self.path} were not read")
        return out

    def read_gds(self, device, names=None) -> dict:
        """Tensors read with GPUDirect Storage (cuFile) straight into device memory, one
        uint8 ``[rows, row_bytes]`` CUDA tensor each, globals first then layer by layer
        (reference ``src/strix/gpu_direct.rs:540-640``). Raises ``OSError`` when cuFile is
        not usable here (see ``gds_available``); callers fall back to ``read_parallel``."""
        from .. import ops
        ext = ops.require_ext()
        if not ext.gds_available():
            raise OSError(f"GPUDirect Storage unavailable: {ext.gds_error()}")
        names = list(self.tensors) if names is None else list(names)
        order = lambda n: (1, int(n.split(".")[1])) if n.startswith("blk.") else (0, 0)
        rd = ext.GdsReader(self.path)
        out = {}
        try:
            for n in sorted(names, key=order):
                t = self.tensors[n]
                buf = torch.empty(t.nbytes, dtype=torch.uint8, device=device)
                got = rd.read(buf, t.offset, t.nbytes, 0)
                if got != t.nbytes:
                    raise OSError(f"short cuFile read of {n}: {got} of {t.nbytes} bytes")
                out[n] = buf.view(t.rows, t.nbytes // t.rows)
        finally:
            rd.close()
        return out

    def dequantize(self, name: str) -> torch.Tensor:
        from .quants import dequantize
        t = self.tensors[name]
        return dequantize(self.raw(name), t.qtype).reshape(t.torch_shape)

    def has(self, name: str) -> bool:
        return name in self.tensors

    def get(self, key: str, default=None):
        return self.metadata.get(key, default)

    def close(self):
        self._buf = None
        if self._mm is not None:
            try:
                self._mm.close()
            except BufferError:
                pass
            self._mm = None

    # -- OS page cache hints (reference: src/weight_streamer.rs:343-389) -----
    def advise(self, name: str, willneed: bool = True):
        t = self.tensors[name]
        if not hasattr(os, "posix_fadvise"):
            return
        fd = os.open(self.path, os.O_RDONLY)
        try:
            os.posix_fadvise(fd, t.offset, t.nbytes,
                             os.POSIX_FADV_WILLNEED if willneed else os.POSIX_FADV_DONTNEED)
        finally:
            os.close(fd)


class _Cursor:
    def __init__(self, mm):
        self.mm = mm
        self.pos = 0

    def unpack(self, fmt: str):
        n = struct.calcsize(fmt)
        v = struct.unpack_from(fmt, self.mm, self.pos)
        self.pos += n
        return v[0] if len(v) == 1 else v

    def string(self) -> str:
        n = self.unpack("<Q")
        s = bytes(self.mm[self.pos:self.pos + n])
        self.pos += n
        return s.decode("utf-8", errors="replace")

    def value(self, vt: int):
        vt = GGUFValueType(vt)
        if vt == GGUFValueType.STRING:
            return self.string()
        if vt == GGUFValueType.ARRAY:
            et = GGUFValueType(self.unpack("<I"))
            n = self.unpack("<Q")
            if et == GGUFValueType.STRING:
                return [self.string() for _ in range(n)]
            if et == GGUFValueType.ARRAY:
                return [self.value(GGUFValueType.ARRAY) for _ in range(n)]
            dt = np.dtype(_NP[et]).newbyteorder("<")
            arr = np.frombuffer(self.mm, dtype=dt, count=n, offset=self.pos).copy()
            self.pos += n * dt.itemsize
            return arr.tolist()
        return self.unpack(_SCALAR[vt])


def read_gguf(path: str | os.PathLike) -> GGUFFile:
    path = os.fspath(path)
    f = open(path, "rb")
    try:
        mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
    finally:
        f.close()
    cur = _Cursor(mm)
    magic = cur.unpack("<I")
    if magic != GGUF_MAGIC:
        raise GGUFError(f"{path}: not a GGUF file (magic {magic:#x})")
    version = cur.unpack("<I")
    if version not in (2, 3):
        raise GGUFError(f"{path}: unsupported GGUF version {version}")
    n_tensors = cur.unpack("<Q")
    n_kv = cur.unpack("<Q")
    metadata: dict[str, Any] = {}
    for _ in range(n_kv):
        key = cur.string()
        vt = cur.unpack("<I")
        metadata[key] = cur.value(vt)
    infos = []
    for _ in range(n_tensors):
        name = cur.string()
        nd = cur.unpack("<I")
        dims = tuple(cur.unpack("<Q") for _ in range(nd))
        qt = GGMLType(cur.unpack("<I"))
        off = cur.unpack("<Q")
        infos.append((name, dims, qt, off))
    alignment = int(metadata.get("general.alignment", GGUF_DEFAULT_ALIGNMENT))
    data_offset = (cur.pos + alignment - 1) // alignment * alignment
    tensors = {}
    for name, dims, qt, off in infos:
        n = 1
        for d in dims:
            n *= d
        nb = tensor_nbytes(qt, n)
        abs_off = data_offset + off
        if abs_off + nb > len(mm):
            raise GGUFError(f"{path}: tensor {name} extends past end of file")
        tensors[name] = TensorInfo(name, dims, qt, abs_off, nb)
    with warnings.catch_warnings():  # read-only mapping: tensors are views we never write
        warnings.simplefilter("ignore", UserWarning)
        buf = torch.frombuffer(memoryview(mm), dtype=torch.uint8) if len(mm) else torch.empty(0, dtype=torch.uint8)
    return GGUFFile(path, version, metadata, tensors, alignment, data_offset, mm, buf)
