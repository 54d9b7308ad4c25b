"""Prefill/decode disaggregation (reference ``src/pd_disagg.rs``, ``src/continuous_batch.rs:256-288``).

Two data planes:

* **GPU (the product path)** — ``PdPair``: the decode engine's KV pool and a flag array live
  in cudaMalloc'd memory that the prefill side maps (same process: peer access; separate
  processes: CUDA IPC via ``air_rs.parallel.symm``-style handles). After the prefill engine
  has filled its own pool for a request, one ``kv_push`` launch copies every
  (layer, block) pair into the blocks the decode side reserved and raises per-pair flags
  there; the decode side enqueues ``kv_wait`` (bounded) on its compute stream, so its first
  decode step reads complete KV without a host round trip. Block ids travel over the host
  control plane.
* **Host connectors** (reference wire format, for cross-node or CPU use): ``KvBlock``
  (4-byte block id, 2-byte layer, 4-byte length, payload; little endian) inside frames that
  add a CRC-32 per block, over TCP (``TcpKvConnector``) or in process (``ShmKvConnector``),
  with per-block int8 quantisation, deadlines (``KvTransferError`` kind "timeout"), checksum
  verification ("corrupt") and in-flight back-pressure ("partial").
"""
from __future__ import annotations

import socket
import struct
import threading
import time
import zlib
from dataclasses import dataclass, field

import torch

# ================================================================================= wire format
HEADER = struct.Struct("<IHI")          # block_id u32, layer u16, data_len u32
FRAME = struct.Struct("<4sQI")          # magic, seq_id u64, n_blocks u32
MAGIC = b"AIRK"

# WARP stream framing (reference ``src/warp_protocol.rs``): every message on a TCP stream is
# [magic "WARP"][version u16][features u64][body_len u32] + body, little endian. The first
# message of a stream is the handshake [model fingerprint 32 B][name_len u16][name]; a body
# length of 0 ends the stream. Same major version required; unknown feature bits rejected.
WARP_MAGIC = b"WARP"
WARP_VERSION = 0x0101
WARP_HEADER = struct.Struct("<4sHQI")
FEAT_LZ4, FEAT_INT8, FEAT_GHOST_PRUNING, FEAT_ASYNC_PIPELINING = 1, 2, 4, 8
WARP_SUPPORTED = FEAT_INT8 | FEAT_ASYNC_PIPELINING


def warp_header(features: int, body_len: int) -> bytes:
    return WARP_HEADER.pack(WARP_MAGIC, WARP_VERSION, features, body_len)


def parse_warp_header(buf: bytes) -> tuple[int, int]:
    """(features, body_len); raises KvTransferError("protocol") on a bad magic, another
    major version or feature bits this side cannot decode."""
    magic, ver, feats, n = WARP_HEADER.unpack(buf)
    if magic != WARP_MAGIC:
        raise KvTransferError("protocol", "bad WARP magic")
    if ver >> 8 != WARP_VERSION >> 8:
        raise KvTransferError("protocol", f"WARP major version {ver >> 8} != {WARP_VERSION >> 8}")
    if feats & ~WARP_SUPPORTED:
        raise KvTransferError("protocol", f"unsupported WARP features {feats & ~WARP_SUPPORTED:#x}")
    return feats, n


def encode_handshake(fingerprint: bytes, name: str) -> bytes:
    nb = name.encode()
    return bytes(fingerprint).ljust(32, b"\0")[:32] + struct.pack("<H", len(nb)) + nb


def decode_handshake(body: bytes) -> tuple[bytes, str]:
    if len(body) < 34:
        raise KvTransferError("protocol", "short WARP handshake")
    (n,) = struct.unpack_from("<H", body, 32)
    if len(body) != 34 + n:
        raise KvTransferError("protocol", "bad WARP handshake length")
    return body[:32], body[34:].decode(errors="replace")


def gguf_fingerprint(path: str) -> bytes:
    """SHA-256 of a GGUF file's header, metadata and tensor table (everything before the
    tensor data) plus its size: two nodes serving the same checkpoint agree on it."""
    import hashlib
    import os
    from ..gguf import read_gguf
    g = read_gguf(path)
    h = hashlib.sha256()
    with open(path, "rb") as f:
        h.update(f.read(g.data_offset))
    h.update(struct.pack("<Q", os.path.getsize(path)))
    return h.digest()


@dataclass
class KvBlock:
    block_id: int
    layer_idx: int
    data: bytes

    def serialise(self) -> bytes:
        return HEADER.pack(self.block_id, self.layer_idx, len(self.data)) + self.data

    @classmethod
    def deserialise(cls, buf: bytes) -> "KvBlock | None":
        if len(buf) < HEADER.size:
            return None
        bid, layer, n = HEADER.unpack_from(buf)
        if len(buf) < HEADER.size + n:
            return None
        return cls(bid, layer, bytes(buf[HEADER.size:HEADER.size + n]))

    @staticmethod
    def int8_quantize(bf16: torch.Tensor) -> tuple[torch.Tensor, float]:
        x = bf16.float()
        amax = float(x.abs().max()) if x.numel() else 0.0
        s = amax / 127.0 if amax > 0 else 1.0
        return torch.round(x / s).clamp(-127, 127).to(torch.int8), s

    @staticmethod
    def int8_dequantize(q: torch.Tensor, s: float) -> torch.Tensor:
        return (q.float() * s).to(torch.bfloat16)


class KvTransferError(Exception):
    def __init__(self, kind: str, msg: str = ""):
        super().__init__(f"{kind}: {msg}" if msg else kind)
        self.kind = kind            # "timeout" | "corrupt" | "partial" | "io"


@dataclass
class TransferMetrics:
    bytes_total: int = 0
    transfers_total: int = 0
    timeouts_total: int = 0
    corrupt_total: int = 0
    latency_sum_us: float = 0.0
    _lock: threading.Lock = field(default_factory=threading.Lock, repr=False)

    def record_transfer(self, nbytes: int, seconds: float):
        with self._lock:
            self.bytes_total += nbytes
            self.transfers_total += 1
            self.latency_sum_us += seconds * 1e6

    def record_timeout(self):
        with self._lock:
            self.timeouts_total += 1

    @property
    def avg_latency_us(self) -> float:
        return self.latency_sum_us / self.transfers_total if self.transfers_total else 0.0


def encode_frame(seq_id: int, blocks: list[KvBlock]) -> bytes:
    out = [FRAME.pack(MAGIC, seq_id, len(blocks))]
    for b in blocks:
        s = b.serialise()
        out.append(s)
        out.append(struct.pack("<I", zlib.crc32(s)))
    return b"".join(out)


def decode_frame(buf: bytes) -> tuple[int, list[KvBlock]]:
    if len(buf) < FRAME.size:
        raise KvTransferError("corrupt", "short frame")
    magic, seq_id, n = FRAME.unpack_from(buf)
    if magic != MAGIC:
        raise KvTransferError("corrupt", "bad magic")
    off, blocks = FRAME.size, []
    for _ in range(n):
        b = KvBlock.deserialise(buf[off:])
        if b is None:
            raise KvTransferError("corrupt", "truncated block")
        end = off + HEADER.size + len(b.data)
        if len(buf) < end + 4 or struct.unpack_from("<I", buf, end)[0] != zlib.crc32(buf[off:end]):
            raise KvTransferError("corrupt", f"checksum mismatch in block {b.block_id}")
        blocks.append(b)
        off = end + 4
    return seq_id, blocks


# ================================================================================= connectors
class ShmKvConnector:
    """In-process connector (single node): frames land in a shared dict."""
    backend_name = "shm"

    def __init__(self):
        self._store: dict[int, list[KvBlock]] = {}
        self._cv = threading.Condition()
        self.drop_next = False            # fault injection: lose the next frame

    def send_blocks(self, seq_id: int, blocks: list[KvBlock], target=None, timeout: float = 2.0) -> int:
        frame = encode_frame(seq_id, blocks)
        if self.drop_next:
            self.drop_next = False
            return len(frame)
        _, got = decode_frame(frame)
        with self._cv:
            self._store.setdefault(seq_id, []).extend(got)
            self._cv.notify_all()
        return len(frame)

    def recv_blocks(self, seq_id: int, n_expected: int, timeout: float = 2.0) -> list[KvBlock]:
        deadline = time.monotonic() + timeout
        with self._cv:
            while len(self._store.get(seq_id, [])) < n_expected:
                left = deadline - time.monotonic()
                if left <= 0:
                    raise KvTransferError("timeout", f"seq {seq_id}: {len(self._store.get(seq_id, []))}/{n_expected}")
                self._cv.wait(left)
            return self._store.pop(seq_id)


class TcpKvConnector:
    """KV frames over TCP in WARP framing, after a model-identity handshake. ``listen()``
    starts the receiver thread."""
    backend_name = "tcp"

    def __init__(self, host: str = "127.0.0.1", port: int = 0, fingerprint: bytes | None = None,
                 model_name: str = ""):
        self.host, self.port = host, port
        # this node's model identity; a receiver with one refuses streams from another model
        self.fingerprint, self.model_name = fingerprint, model_name
        self.peers: list[tuple[bytes, str]] = []
        self._store: dict[int, list[KvBlock]] = {}
        self._errors: list[KvTransferError] = []
        self._cv = threading.Condition()
        self._srv: socket.socket | None = None

    def listen(self) -> int:
        self._srv = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
        self._srv.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
        self._srv.bind((self.host, self.port))
        self._srv.listen(16)
        self.port = self._srv.getsockname()[1]
        threading.Thread(target=self._accept_loop, daemon=True).start()
        return self.port

    def _accept_loop(self):
        while True:
            try:
                conn, _ = self._srv.accept()
            except OSError:
                return
            threading.Thread(target=self._serve, args=(conn,), daemon=True).start()

    @staticmethod
    def _read_exact(conn, n):
        buf = bytearray()
        while len(buf) < n:
            chunk = conn.recv(n - len(buf))
            if not chunk:
                raise KvTransferError("io", "connection closed")
            buf += chunk
        return bytes(buf)

    def _serve(self, conn):
        with conn:
            try:
                _, n = parse_warp_header(self._read_exact(conn, WARP_HEADER.size))
                fp, name = decode_handshake(self._read_exact(conn, n))
                if self.fingerprint is not None and fp != bytes(self.fingerprint).ljust(32, b"\0")[:32]:
                    raise KvTransferError("handshake", f"KV stream from another model ({name!r})")
                with self._cv:
                    self.peers.append((fp, name))
                while True:
                    try:
                        hdr = self._read_exact(conn, WARP_HEADER.size)
                    except KvTransferError:
                        return
                    _, n = parse_warp_header(hdr)
                    if n == 0:                             # end of stream
                        return
                    seq_id, blocks = decode_frame(self._read_exact(conn, n))
                    with self._cv:
                        self._store.setdefault(seq_id, []).extend(blocks)
                        self._cv.notify_all()
            except KvTransferError as e:
                with self._cv:
                    self._errors.append(e)
                    self._cv.notify_all()

    def send_blocks(self, seq_id: int, blocks: list[KvBlock], target, timeout: float = 2.0,
                    corrupt: bool = False, features: int = 0) -> int:
        """``features``: WARP bits of the payload (FEAT_INT8 for ``blocks_from_pool(quantize=True)``)."""
        frame = bytearray(encode_frame(seq_id, blocks))
        if corrupt and len(frame) > FRAME.size + HEADER.size:   # fault injection: flip a payload bit
            frame[FRAME.size + HEADER.size] ^= 0x01
        try:
            hs = encode_handshake(self.fingerprint or b"", self.model_name)
            with socket.create_connection(target, timeout=timeout) as s:
                s.sendall(warp_header(0, len(hs)) + hs)
                s.sendall(warp_header(features, len(frame)) + bytes(frame))
                s.sendall(warp_header(0, 0))
        except OSError as e:
            raise KvTransferError("io", str(e))
        return len(frame)

    def recv_blocks(self, seq_id: int, n_expected: int, timeout: float = 2.0) -> list[KvBlock]:
        deadline = time.monotonic() + timeout
        with self._cv:
            while len(self._store.get(seq_id, [])) < n_expected:
                if self._errors:
                    raise self._errors.pop(0)
                left = deadline - time.monotonic()
                if left <= 0:
                    raise KvTransferError("timeout", f"seq {seq_id}")
                self._cv.wait(left)
            return self._store.pop(seq_id)

    def close(self):
        if self._srv is not None:
            self._srv.close()


@dataclass
class PdDisaggConfig:
    prefill_addr: tuple[str, int] = ("127.0.0.1", 9100)
    decode_addr: tuple[str, int] = ("127.0.0.1", 9101)
    max_in_flight: int = 16
    transfer_timeout: float = 2.0


def blocks_from_pool(kv: torch.Tensor, block_ids: list[int], quantize: bool = True) -> list[KvBlock]:
    """Host KvBlocks (per layer, per block) of a paged pool kv [L, nb, 2, nkv, bs, d]."""
    out = []
    for l in range(kv.shape[0]):
        for b in block_ids:
            t = kv[l, b].contiguous().cpu()
            if quantize:
                q, s = KvBlock.int8_quantize(t)
                data = struct.pack("<f", s) + q.numpy().tobytes()
            else:
                data = t.view(torch.uint8).numpy().tobytes()
            out.append(KvBlock(b, l, data))
    return out


def blocks_into_pool(kv: torch.Tensor, blocks: list[KvBlock], id_map: dict[int, int], quantize: bool = True):
    shape = tuple(kv.shape[2:])
    for blk in blocks:
        if quantize:
            (s,) = struct.unpack_from("<f", blk.data)
            q = torch.frombuffer(bytearray(blk.data[4:]), dtype=torch.int8).reshape(shape)
            t = KvBlock.int8_dequantize(q, s)
        else:
            t = torch.frombuffer(bytearray(blk.data), dtype=torch.uint8).view(torch.bfloat16).reshape(shape)
        kv[blk.layer_idx, id_map[blk.block_id]] = t.to(kv.device)


class PrefillNode:
    """Sends a finished prefill's KV blocks; refuses beyond ``max_in_flight`` transfers."""

    def __init__(self, cfg: PdDisaggConfig, connector):
        self.cfg, self.connector, self.metrics = cfg, connector, TransferMetrics()
        self._inflight = 0
        self._lock = threading.Lock()

    def prefill_and_send(self, seq_id: int, kv: torch.Tensor, block_ids: list[int], quantize: bool = True) -> int:
        with self._lock:
            if self._inflight >= self.cfg.max_in_flight:
                raise KvTransferError("partial", "too many transfers in flight")
            self._inflight += 1
        t0 = time.perf_counter()
        try:
            blocks = blocks_from_pool(kv, block_ids, quantize)
            n = self.connector.send_blocks(seq_id, blocks, self.cfg.decode_addr, self.cfg.transfer_timeout)
            self.metrics.record_transfer(n, time.perf_counter() - t0)
            return len(blocks)
        finally:
            with self._lock:
                self._inflight -= 1


class DecodeNode:
    def __init__(self, cfg: PdDisaggConfig, connector):
        self.cfg, self.connector, self.metrics = cfg, connector, TransferMetrics()

    def recv_and_prepare(self, seq_id: int, kv: torch.Tensor, id_map: dict[int, int], n_layers: int,
                         quantize: bool = True) -> int:
        t0 = time.perf_counter()
        try:
            blocks = self.connector.recv_blocks(seq_id, n_layers * len(id_map), self.cfg.transfer_timeout)
        except KvTransferError as e:
            if e.kind == "timeout":
                self.metrics.record_timeout()
            raise
        blocks_into_pool(kv, blocks, id_map, quantize)
        self.metrics.record_transfer(sum(len(b.data) for b in blocks), time.perf_counter() - t0)
        return len(blocks)


# ================================================================================= GPU path
class KvPushLink:
    """Device-side prefill->decode KV copy into a (possibly peer / IPC-mapped) decode pool."""

    def __init__(self, dst_kv_ptr: int, dst_shape: tuple, flags_ptr: int, device, timeout_s: float = 2.0,
                 elem_size: int = 2):
        self.dst = dst_kv_ptr
        self.dst_shape = dst_shape                   # (L, nb, 2, nkv, bs, row elements)
        self.elem_size = elem_size                   # 2: bf16 pool, 1: fp8 pool (uint8 rows)
        self.flags = flags_ptr
        self.device = torch.device(device)
        self.timeout_s = timeout_s
        self.tag = 0
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)

    @staticmethod
    def block_bytes(shape, elem_size: int = 2) -> int:
        n = elem_size
        for d in shape[2:]:
            n *= d
        return n

    def push(self, src_kv: torch.Tensor, src_blocks: list[int], dst_blocks: list[int]) -> int:
        """Enqueue the copy on the current stream; returns the transfer tag."""
        from .. import ops
        ext = ops.require_ext()
        self.tag += 1
        L, nb = self.dst_shape[0], self.dst_shape[1]
        bb = self.block_bytes(self.dst_shape, self.elem_size)
        assert tuple(src_kv.shape[2:]) == tuple(self.dst_shape[2:]) and src_kv.shape[0] == L
        assert src_kv.element_size() == self.elem_size, "prefill and decode pools differ in KV dtype"
        sb = torch.tensor(src_blocks, dtype=torch.int32, device=src_kv.device)
        db = torch.tensor(dst_blocks, dtype=torch.int32, device=src_kv.device)
        ext.kv_push(src_kv.data_ptr(), src_kv.stride(0) * self.elem_size, src_kv.shape[1], self.dst, nb * bb, nb, bb, L,
                    sb, db, self.flags, nb, self.tag, self.err)
        ops.count_launch()
        return self.tag


def kv_wait(flags: torch.Tensor, dst_blocks: list[int], n_layers: int, tag: int, timeout_s: float = 2.0):
    """Enqueue the bounded flag wait on the decode side's current stream; returns the
    status tensor (0 = all blocks arrived, 2 = timed out)."""
    from .. import ops
    status = torch.zeros(1, dtype=torch.int32, device=flags.device)
    db = torch.tensor(dst_blocks, dtype=torch.int32, device=flags.device)
    ops.require_ext().kv_wait(flags.data_ptr(), flags.shape[-1], db, n_layers, tag, timeout_s, status)
    ops.count_launch()
    return status


class PdPair:
    """A prefill engine and a decode engine in one process (one GPU, or two GPUs with peer
    access) joined by the device KV push; across processes the decode pool and flags are
    exported with CUDA IPC (``air_rs._C.ipc_handle``/``ipc_open``) and ``KvPushLink`` takes
    the mapped addresses."""

    def __init__(self, prefill, decode, timeout_s: float = 2.0):
        from .. import ops
        self.p, self.d = prefill, decode
        ext = ops.require_ext()
        dd, pd_ = decode.runner.device, prefill.runner.device
        if dd != pd_:
            if not ext.enable_peer_access(pd_.index, dd.index):
                raise RuntimeError(f"no peer access from {pd_} to {dd}")
        nb = decode.runner.kv.shape[1]
        self.flags = torch.zeros(decode.runner.kv.shape[0], nb, dtype=torch.int32, device=dd)
        self.link = KvPushLink(decode.runner.kv.data_ptr(), tuple(decode.runner.kv.shape), self.flags.data_ptr(),
                               pd_, timeout_s, elem_size=decode.runner.kv.element_size())
        self.timeout_s = timeout_s
        self.metrics = TransferMetrics()

    def submit(self, prompt_ids: list[int], params, verify: bool = False) -> int:
        """Prefill on the prefill engine, push its KV into the decode engine, and hand the
        request over (its first token already sampled). Returns the decode-side rid."""
        p, d = self.p, self.d
        with torch.cuda.device(p.runner.device):
            rid = p.add_request(prompt_ids, params)
            r = p.waiting[-1]
            adm = p._admit()
            assert r in adm, "prefill engine could not admit the request"
            p._prefill(adm)
        first = r.output_ids[0]
        src_blocks = p.seqs.block_table(r.seq)
        # decode side: reserve the same number of tokens' blocks
        with torch.cuda.device(d.runner.device):
            dr = d._request_for_handoff(r.prompt_ids, params, [first])
        dst_blocks = d.seqs.block_table(dr.seq)
        t0 = time.perf_counter()
        ev = torch.cuda.Event()
        with torch.cuda.device(p.runner.device):
            tag = self.link.push(p.runner.kv, src_blocks, dst_blocks)
            ev.record()
        with torch.cuda.device(d.runner.device):
            torch.cuda.current_stream().wait_event(ev)
            status = kv_wait(self.flags, dst_blocks, d.runner.kv.shape[0], tag, self.timeout_s)
        if int(status.item()) != 0 or int(self.link.err.item()) != 0:
            self.metrics.record_timeout()
            with torch.cuda.device(d.runner.device):
                d.abort(dr.rid)
            raise KvTransferError("timeout", f"KV push for request {rid} did not complete")
        if verify:   # debugging aid: the decode pool now holds exactly the prefill KV
            a_ = p.runner.kv[:, torch.tensor(src_blocks, device=p.runner.device)].cpu()
            b_ = d.runner.kv[:, torch.tensor(dst_blocks, device=d.runner.device)].cpu()
            if not torch.equal(a_, b_):
                raise KvTransferError("corrupt", f"decode blocks differ from prefill blocks "
                                                 f"({int((a_ != b_).sum())} elements)")
        self.metrics.record_transfer(len(src_blocks) * d.runner.kv.shape[0] * KvPushLink.block_bytes(
            tuple(d.runner.kv.shape), d.runner.kv.element_size()), time.perf_counter() - t0)
        with torch.cuda.device(p.runner.device):
            p.abort(rid)               # the prefill side's copy is no longer needed
        return dr.rid
