"""Fused tensor-parallel all-reduce over NVLink peer memory (reference: the host TCP ring
all-reduce after the row-parallel O and down projections, ``src/model.rs:596-607,728-739``,
``src/distributed.rs``).

Each rank cudaMallocs one receive buffer (``[2 parities][world][slot]`` of 8-byte
(value, tag) elements), exports a CUDA IPC handle, and maps every peer's buffer into its
own address space. The row-parallel projection pushes every finished output element into
every rank's buffer as one tagged 8-byte store (the GEMV epilogue ``EPI_PEER_PUSH``, or
``peer_push`` after the tcgen05 GEMM); the following RMSNorm (``reduce_rmsnorm_quant``)
waits per element for this collective's tag in its local buffer, sums the partials into
the residual stream and quantises the normalised row for the next GEMV. All state is
device-resident (epoch counter, tags), so the sequence is CUDA-graph capturable.

``PeerComm.local_group`` builds W communicators on one GPU whose "peer" buffers are local
allocations: the same kernels run with every rank's data in one process, which is how the
protocol is tested with fewer GPUs than ranks (producers never wait, so running the ranks'
launches one after another on one stream is always safe).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops
from .tp import COMM, TPGroup

MAX_PEERS = 8
DEFAULT_TIMEOUT_S = 2.0


class PeerComm:
    def __init__(self, bases: list[int], rank: int, device, slot_elems: int, owned: list,
                 timeout_s: float = DEFAULT_TIMEOUT_S):
        self.world = len(bases)
        if not 1 <= self.world <= MAX_PEERS:
            raise ValueError(f"peer all-reduce supports 1..{MAX_PEERS} ranks")
        self.rank, self.device = rank, torch.device(device)
        self.slot_elems = slot_elems
        self._owned = owned                       # keeps buffers / IPC mappings alive
        self.epoch = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.done = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        pm = [0] * 12
        pm[:len(bases)] = bases
        pm[8], pm[9], pm[10], pm[11] = self.epoch.data_ptr(), slot_elems, self.world, rank
        self.push_meta = torch.tensor(pm, dtype=torch.int64)
        self.reduce_meta = torch.tensor([bases[rank], self.epoch.data_ptr(), self.done.data_ptr(),
                                         self.err.data_ptr(), slot_elems, self.world, int(timeout_s * 1e9)],
                                        dtype=torch.int64)
        self.pending = False

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
        comm = cls(bases, tp.rank, dev, slot, [buf], timeout_s)
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
        return [cls(bases, r, dev, slot, bufs, timeout_s) for r in range(world)]

    def close(self):
        ext = ops.require_ext()
        for p in getattr(self, "_opened", []):
            ext.ipc_close(p)
        self._opened = []

    # ----------------------------------------------------------------- producer side
    def fits(self, B: int, N: int) -> bool:
        return B * N <= self.slot_elems

    def push_gemv(self, w: ops.QWeight, xq, xds, B: int, err=None):
        """Row-parallel decode GEMV whose epilogue pushes the partial to every rank."""
        ops.gemv(w, xq, xds, B, ops.EPI_PEER_PUSH, ld_out=w.N, push_meta=self.push_meta, err=err)
        COMM.record("peer_push", B * w.N * 4 * (self.world - 1))
        self.pending = True

    def push(self, src: torch.Tensor, B: int):
        """Push an fp32 partial [B, N] computed by another kernel."""
        ops.require_ext().peer_push(self.push_meta, src, B, src.shape[1], src.stride(0))
        ops.count_launch()
        COMM.record("peer_push", B * src.shape[1] * 4 * (self.world - 1))
        self.pending = True

    # ----------------------------------------------------------------- consumer side
    def reduce_norm(self, x, w, eps: float, xq=None, xds=None, y_bf16=None, B: int | None = None,
                    w_offset: float = 0.0):
        """x += sum of all ranks' pushed partials, then RMSNorm (+ Q8A quantisation)."""
        B = B if B is not None else x.shape[0]
        K = x.shape[1]
        ops.require_ext().reduce_rmsnorm_quant(self.reduce_meta, x, w, w_offset, eps, B, K, xq, xds, y_bf16)
        ops.count_launch()
        self.pending = False

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
    """Wrap an NCCL TPGroup with the peer-memory all-reduce (impl "ours"); "nccl" keeps NCCL."""
    if tp is None or impl == "nccl" or hidden is None:
        return tp
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    return FusedTP(tp, PeerComm.create(tp, max_rows, hidden, dev))
