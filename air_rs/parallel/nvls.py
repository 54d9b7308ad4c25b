"""Tensor-parallel all-reduce through NVLink SHARP (NVLS) multicast memory.

The same place in the decode step as ``PeerComm`` (the sum after the row-parallel O and
down projections, reference ``src/model.rs:596-607,728-739``), with the reduction done by
the NVSwitch instead of by every rank:

* the buffer is a symmetric allocation (``torch.distributed._symmetric_memory``) bound to a
  multicast object: ``[2 parities][rows][hidden]`` fp32 partials, then ``[2][rows][world]``
  int32 row-arrival flags;
* the producer (decode GEMV or tcgen05 GEMM, plain store epilogue) writes this rank's
  partial into its own copy of the parity's region: local stores only;
* the consumer (``tp_reduce_norm_nvls``) CTA of row b stores the collective's tag into row
  b's flag on every rank, waits (bounded) for every rank's flag, then reads the row with
  ``multimem.ld_reduce.add.f32`` on the multicast address: the switch returns the sum of
  every rank's partial, which is added to the residual stream and normalised / quantised in
  the same pass (RMSNorm or LayerNorm, Q8A and/or bf16 out).

Parities alternate per collective on the host (static per captured CUDA graph: a decode step
has two collectives per layer, an even count). Collective i writes parity i % 2; a rank
reaches collective i only after its collective i - 1 saw every rank's flag, so every rank
has finished reading parity i % 2 of collective i - 2 by then. Flags carry the local epoch
(+1), which every rank advances identically, so no flag is ever reset.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops
from .tp import COMM, TPGroup

MAX_PEERS = 8
DEFAULT_TIMEOUT_S = 2.0


def nvls_available(tp: TPGroup) -> bool:
    """Multicast objects need CUDA GPUs joined by NVSwitch and the symmetric-memory module."""
    try:
        import torch.distributed._symmetric_memory  # noqa: F401
    except ImportError:
        return False
    return tp is not None and tp.world_size > 1 and torch.cuda.is_available()


class NvlsComm:
    """One rank's NVLS all-reduce state (interface of ``PeerComm``: fits / push_gemv /
    push_gemm / push / reduce_norm / check / close)."""

    def __init__(self, buf: torch.Tensor, handle, rank: int, world: int, device, max_rows: int, hidden: int,
                 timeout_s: float = DEFAULT_TIMEOUT_S):
        self.buf, self.handle = buf, handle
        self.rank, self.world, self.device = rank, world, torch.device(device)
        self.max_rows, self.hidden = max_rows, hidden
        self.slot_elems = max_rows * hidden
        self.epoch = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.done = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        data_bytes = 2 * self.slot_elems * 4
        flag_bytes = max_rows * world * 4
        self.slots = [buf[p * self.slot_elems * 4:(p + 1) * self.slot_elems * 4].view(torch.float32)
                      .view(max_rows, hidden) for p in range(2)]
        mc = int(handle.multicast_ptr)
        peers = [int(x) for x in handle.buffer_ptrs]
        local = buf.data_ptr()
        self.metas = []
        for p in range(2):
            foff = data_bytes + p * flag_bytes
            fpeer = [b + foff for b in peers] + [0] * (MAX_PEERS - world)
            self.metas.append(torch.tensor(
                [mc + p * self.slot_elems * 4, local + foff] + fpeer +
                [self.epoch.data_ptr(), self.done.data_ptr(), self.err.data_ptr(), world, rank,
                 int(timeout_s * 1e9), self.slot_elems], dtype=torch.int64))
        self.parity = 0
        self.pending = False

    @staticmethod
    def buffer_bytes(max_rows: int, hidden: int, world: int) -> int:
        return 2 * max_rows * hidden * 4 + 2 * max_rows * world * 4

    @classmethod
    def create(cls, tp: TPGroup, max_rows: int, hidden: int, device, timeout_s: float = DEFAULT_TIMEOUT_S):
        """Collective: every rank of ``tp`` calls this. Raises RuntimeError when the GPUs
        offer no multicast object (no NVSwitch / NVLS)."""
        import torch.distributed._symmetric_memory as symm
        dev = torch.device(device)
        group = tp.group if tp.group is not None else dist.group.WORLD
        name = group.group_name
        try:
            symm.enable_symm_mem_for_group(name)
        except Exception:  # noqa: BLE001 - newer releases enable every group
            pass
        buf = symm.empty(cls.buffer_bytes(max_rows, hidden, tp.world_size), dtype=torch.uint8, device=dev)
        buf.zero_()
        torch.cuda.synchronize(dev)
        handle = symm.rendezvous(buf, name)
        ok = torch.tensor([1 if int(getattr(handle, "multicast_ptr", 0) or 0) != 0 else 0], device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=tp.group)
        if int(ok.item()) == 0:
            raise RuntimeError("NVLS: no multicast object on this GPU group")
        comm = cls(buf, handle, tp.rank, tp.world_size, dev, max_rows, hidden, timeout_s)
        dist.barrier(group=tp.group)          # every buffer is zeroed before any flag is raised
        return comm

    def close(self):
        """Every rank must be idle (synchronised and past a barrier) before this is called."""
        self.handle = None
        self.buf = None
        self.slots = []

    # ----------------------------------------------------------------- producer side
    def two_shot(self, B: int) -> bool:
        return False

    def fits(self, B: int, N: int) -> bool:
        return N == self.hidden and B <= self.max_rows

    def _slot(self, B: int) -> torch.Tensor:
        return self.slots[self.parity][:B]

    def _record(self, B: int):
        # bytes this rank's partial contributes to the switch reduction (read once) and the
        # reduced row it reads back
        COMM.record("nvls_allreduce", 2 * B * self.hidden * 4)
        self.pending = True

    def push_gemv(self, w: ops.QWeight, xq, xds, B: int, err=None):
        """Row-parallel decode GEMV storing its fp32 partial into this rank's symmetric slot."""
        ops.gemv(w, xq, xds, B, ops.EPI_STORE, out_f32=self._slot(B), ld_out=w.N, err=err)
        self._record(B)

    def push_gemm(self, x_bf16, w: ops.QWeight, dummy_out, err=None):
        """Row-parallel tcgen05 GEMM storing its fp32 partial into this rank's symmetric slot."""
        from ..ops import gemm
        B = x_bf16.shape[0]
        gemm.linear(x_bf16, w, self._slot(B), err=err)
        self._record(B)

    def push(self, src: torch.Tensor, B: int):
        """An fp32 partial [B, N] computed by another kernel."""
        self._slot(B).copy_(src[:B])
        self._record(B)

    # ----------------------------------------------------------------- consumer side
    def reduce_norm(self, x, w, eps: float, xq=None, xds=None, y_bf16=None, B: int | None = None,
                    w_offset: float = 0.0, bias=None, layer: bool = False):
        """x += the switch-reduced sum of every rank's partial, then RMSNorm / LayerNorm (+ Q8A)."""
        B = B if B is not None else x.shape[0]
        ops.require_ext().tp_reduce_norm_nvls(self.metas[self.parity], x, w, w_offset, eps, B, x.shape[1],
                                              xq, xds, y_bf16, bias, int(layer))
        ops.count_launch()
        self.parity ^= 1
        self.pending = False

    def check(self):
        if int(self.err.item()) != 0:
            raise RuntimeError(f"NVLS all-reduce: a wait for a peer's row flag timed out (code {int(self.err.item())})")
