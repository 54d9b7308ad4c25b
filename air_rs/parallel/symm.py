"""Fused tensor-parallel all-reduce over NVLink peer memory (reference: the host TCP ring
all-reduce after the row-parallel O and down projections, ``src/model.rs:596-607,728-739``,
``src/distributed.rs``).

Each rank cudaMallocs one receive buffer (partials ``[2 parities][world][slot]`` then an
all-gather region ``[2][slot]``, 8-byte (value, tag) elements), exports a CUDA IPC handle,
and maps every peer's buffer into its own address space. The row-parallel projection
stores every finished output element over NVLink as one tagged 8-byte store, from the
decode GEMV epilogue (``EPI_PEER_PUSH``), the tcgen05 GEMM epilogue (``GEMM_PEER_PUSH``), or
``peer_push`` after another kernel; the following RMSNorm (``tp_reduce_norm``) waits per
element for this collective's tag in its local buffer, sums into the residual stream and
quantises the normalised row for the next projection. All state is device-resident (epoch
counter, tags), so the sequence is CUDA-graph capturable.

Two data paths, picked per collective from the row count (``two_shot``):
* one-shot: every rank's whole partial goes to every rank (one hop; (world-1) x the bytes);
* two-shot: column c goes only to its owner rank (reduce-scatter), the owner adds the
  residual and writes the new values into every rank's all-gather region (two hops;
  2 (world-1) / world x the bytes). At 8 GPUs that is 4x fewer bytes per rank.

``PeerComm.local_group`` builds W communicators on one GPU whose "peer" buffers are local
allocations; ``reduce_norm_group`` runs every rank's consumer in one launch. That is how
the protocol is tested with fewer GPUs than ranks: producers never wait, and the consumers
that wait on one another run as CTAs of one launch, never as separate launches.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops
from .tp import COMM, TPGroup

MAX_PEERS = 8
DEFAULT_TIMEOUT_S = 2.0


GEMM_PEER_PUSH = 3


class PeerComm:
    def __init__(self, bases: list[int], rank: int, device, slot_elems: int, owned: list, hidden: int,
                 timeout_s: float = DEFAULT_TIMEOUT_S):
        self.world = len(bases)
        if not 1 <= self.world <= MAX_PEERS:
            raise ValueError(f"peer all-reduce supports 1..{MAX_PEERS} ranks")
        self.rank, self.device = rank, torch.device(device)
        self.slot_elems, self.hidden = slot_elems, hidden
        self.max_rows = slot_elems // hidden
        # columns owned per rank on the two-shot path: a multiple of 32 (one Q8A group)
        self.shard = -(-hidden // (32 * self.world)) * 32
        self._owned = owned                       # keeps buffers / IPC mappings alive
        self.epoch = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.done = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        ag_off = 2 * self.world * slot_elems * 8          # bytes to the all-gather region

        def push_meta(shard):
            pm = [0] * 14
            pm[:len(bases)] = bases
            pm[8], pm[9], pm[10], pm[11] = self.epoch.data_ptr(), slot_elems, self.world, rank
            pm[12], pm[13] = hidden, shard
            return torch.tensor(pm, dtype=torch.int64)
        self.push_meta_one = push_meta(0)
        self.push_meta_two = push_meta(self.shard)
        ag_peer = [b + ag_off for b in bases] + [0] * (MAX_PEERS - len(bases))
        self.reduce_meta = torch.tensor(
            [bases[rank], bases[rank] + ag_off] + ag_peer +
            [self.epoch.data_ptr(), self.done.data_ptr(), self.err.data_ptr(), slot_elems, self.world, rank,
             int(timeout_s * 1e9), self.shard], dtype=torch.int64)
        import os
        # rows from which the two-shot path is used (it needs all consumer CTAs resident)
        self.two_shot_min_rows = int(os.environ.get("AIR_TP_TWO_SHOT_MIN_ROWS", "9"))
        self.pending = False

    def two_shot(self, B: int) -> bool:
        return self.world > 2 and self.two_shot_min_rows <= B <= 148

    def push_meta(self, B: int) -> torch.Tensor:
        return self.push_meta_two if self.two_shot(B) else self.push_meta_one

    # ----------------------------------------------------------------- construction

    @classmethod
    def create(cls, tp: TPGroup, max_rows: int, hidden: int, device, timeout_s: float = DEFAULT_TIMEOUT_S):
        """Collective: every rank of ``tp`` calls this; exchanges IPC handles."""
        ext = ops.require_ext()
        dev = torch.device(device)
        slot = max_rows * hidden
        buf = ext.comm_alloc(ext.peer_buffer_bytes(tp.world_size, slot), dev.index or 0)
        handles = [None] * tp.world_size
        dist.all_gather_object(handles, ext.ipc_handle(buf), group=tp.group)
        bases, opened = [], []
        for r, h in enumerate(handles):
            if r == tp.rank:
                bases.append(buf.data_ptr())
            else:
                p = ext.ipc_open(h, dev.index or 0)
                opened.append(p)
                bases.append(p)
        comm = cls(bases, tp.rank, dev, slot, [buf], hidden, timeout_s)
        comm._opened = opened
        torch.cuda.synchronize(dev)
        dist.barrier(group=tp.group)             # every buffer is zeroed before any push
        return comm

    @classmethod
    def local_group(cls, world: int, max_rows: int, hidden: int, device, timeout_s: float = DEFAULT_TIMEOUT_S):
        """``world`` communicators on one GPU (all buffers local); see the module docstring."""
        ext = ops.require_ext()
        dev = torch.device(device)
        slot = max_rows * hidden
        bufs = [ext.comm_alloc(ext.peer_buffer_bytes(world, slot), dev.index or 0) for _ in range(world)]
        bases = [b.data_ptr() for b in bufs]
        return [cls(bases, r, dev, slot, bufs, hidden, timeout_s) for r in range(world)]

    def close(self):
        ext = ops.require_ext()
        for p in getattr(self, "_opened", []):
            ext.ipc_close(p)
        self._opened = []

    # ----------------------------------------------------------------- producer side
    def fits(self, B: int, N: int) -> bool:
        return N == self.hidden and B <= self.max_rows

    def _bytes_out(self, B: int) -> int:
        """Bytes this rank stores over NVLink for one collective of B rows."""
        n = B * self.hidden * 8
        if self.two_shot(B):
            return 2 * n * (self.world - 1) // self.world
        return n * (self.world - 1)

    def push_gemv(self, w: ops.QWeight, xq, xds, B: int, err=None):
        """Row-parallel decode GEMV whose epilogue pushes the partial over NVLink."""
        ops.gemv(w, xq, xds, B, ops.EPI_PEER_PUSH, ld_out=w.N, push_meta=self.push_meta(B), err=err)
        COMM.record("peer_push", self._bytes_out(B))
        self.pending = True

    def push_gemm(self, x_bf16, w: ops.QWeight, dummy_out, err=None):
        """Row-parallel tcgen05 GEMM whose epilogue pushes the partial over NVLink."""
        from ..ops import gemm
        B = x_bf16.shape[0]
        gemm.linear(x_bf16, w, dummy_out, err=err, push_meta=self.push_meta(B))
        COMM.record("peer_push", self._bytes_out(B))
        self.pending = True

    def push(self, src: torch.Tensor, B: int):
        """Push an fp32 partial [B, N] computed by another kernel."""
        ops.require_ext().peer_push(self.push_meta(B), src, B, src.shape[1], src.stride(0))
        ops.count_launch()
        COMM.record("peer_push", self._bytes_out(B))
        self.pending = True

    # ----------------------------------------------------------------- consumer side
    def reduce_norm(self, x, w, eps: float, xq=None, xds=None, y_bf16=None, B: int | None = None,
                    w_offset: float = 0.0, bias=None, layer: bool = False):
        """x += sum of all ranks' pushed partials, then RMSNorm / LayerNorm (+ Q8A quantisation)."""
        B = B if B is not None else x.shape[0]
        K = x.shape[1]
        ops.require_ext().tp_reduce_norm([self.reduce_meta], [x], w, w_offset, eps, B, K,
                                         [xq] if xq is not None else [], [xds] if xds is not None else [],
                                         [y_bf16] if y_bf16 is not None else [], self.two_shot(B),
                                         bias, int(layer))
        ops.count_launch()
        self.pending = False

    @staticmethod
    def reduce_norm_group(comms: list["PeerComm"], xs, w, eps: float, xqs=None, xdss=None, ys=None,
                          B: int | None = None, w_offset: float = 0.0, bias=None, layer: bool = False):
        """Every rank's ``reduce_norm`` of a ``local_group`` in one launch (one GPU)."""
        B = B if B is not None else xs[0].shape[0]
        K = xs[0].shape[1]
        ops.require_ext().tp_reduce_norm([c.reduce_meta for c in comms], list(xs), w, w_offset, eps, B, K,
                                         list(xqs or []), list(xdss or []), list(ys or []),
                                         comms[0].two_shot(B), bias, int(layer))
        ops.count_launch()
        for c in comms:
            c.pending = False

    def check(self):
        if int(self.err.item()) != 0:
            raise RuntimeError(f"peer all-reduce: a wait for peer data timed out (code {int(self.err.item())})")


class FusedTP(TPGroup):
    """TPGroup whose decode all-reduces run through ``PeerComm``; NCCL stays for the rest
    (prefill chunks larger than the receive slot, the vocab all-gather)."""

    def __init__(self, tp: TPGroup, peer: PeerComm):
        self.__dict__.update(tp.__dict__)
        self.peer = peer


def maybe_fused_tp(tp, impl: str = "ours", max_rows: int = 64, hidden: int | None = None, device=None):
    """Wrap an NCCL TPGroup with the peer-memory all-reduce (impl "ours") or the NVLink SHARP
    multicast all-reduce (impl "nvls", ``air_rs.parallel.nvls``); "nccl" keeps NCCL."""
    if tp is None or impl == "nccl" or hidden is None:
        return tp
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    if impl == "nvls":
        from .nvls import NvlsComm
        return FusedTP(tp, NvlsComm.create(tp, max_rows, hidden, dev))
    return FusedTP(tp, PeerComm.create(tp, max_rows, hidden, dev))
