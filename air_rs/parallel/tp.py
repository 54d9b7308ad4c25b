"""Tensor parallelism (Megatron column/row split) across one process per GPU.

Column-parallel: QKV heads and gate/up rows are split across ranks; row-parallel: O and
down are split along their input dim in whole quant blocks (the reference dequantises to
F16 and narrows, ``src/tensor_parallel.rs:104-161``; here shards stay quantised). The
partial outputs are summed across ranks after O and down (the reference does this over a
host TCP ring, ``src/model.rs:596-607,728-739``), and the vocab-parallel LM head's logits
are gathered before sampling.

``TPGroup`` is the NCCL baseline data plane. ``air_rs.parallel.symm.FusedTP`` replaces its
all-reduce with the fused peer-memory kernel on NVLink.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class CommStats:
    """Calls and payload bytes per collective kind, process-wide. Payload bytes are what one
    rank contributes: the partial it all-reduces, the shard it all-gathers, the rows it pushes
    to each peer. Collectives inside a CUDA graph are recorded once at capture and added per
    replay by the runner (``snapshot`` / ``since`` / ``add``)."""

    def __init__(self):
        self.calls: dict[str, int] = {}
        self.bytes: dict[str, int] = {}

    def record(self, kind: str, nbytes: int, calls: int = 1):
        self.calls[kind] = self.calls.get(kind, 0) + calls
        self.bytes[kind] = self.bytes.get(kind, 0) + int(nbytes)

    def snapshot(self) -> dict[str, tuple[int, int]]:
        return {k: (self.calls[k], self.bytes[k]) for k in self.calls if self.calls[k] or self.bytes[k]}

    def since(self, snap: dict[str, tuple[int, int]]) -> dict[str, tuple[int, int]]:
        now = self.snapshot()
        return {k: (c - snap.get(k, (0, 0))[0], b - snap.get(k, (0, 0))[1]) for k, (c, b) in now.items()
                if (c, b) != snap.get(k, (0, 0))}

    def add(self, delta: dict[str, tuple[int, int]], sign: int = 1):
        for k, (c, b) in delta.items():
            self.record(k, sign * b, sign * c)

    def totals(self) -> tuple[int, int]:
        return sum(self.calls.values()), sum(self.bytes.values())

    def reset(self):
        self.calls.clear()
        self.bytes.clear()


COMM = CommStats()


class TPGroup:
    def __init__(self, group=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world_size = dist.get_world_size(group)
        self._gather_buf: torch.Tensor | None = None

    def all_reduce_add(self, partial: torch.Tensor, x: torch.Tensor):
        """x += sum over ranks of partial (fp32)."""
        dist.all_reduce(partial, group=self.group)
        COMM.record("all_reduce", partial.numel() * partial.element_size())
        x.add_(partial)

    def all_gather_vocab(self, local: torch.Tensor, full: torch.Tensor) -> torch.Tensor:
        """[B, V_l] shards -> [B, V] (the last shard may be padded)."""
        B, Vl = local.shape
        W = self.world_size
        n = W * B * Vl
        if self._gather_buf is None or self._gather_buf.numel() < n:
            self._gather_buf = torch.empty(n, dtype=local.dtype, device=local.device)
        buf = self._gather_buf[:n].view(W, B, Vl)
        dist.all_gather_into_tensor(buf.view(W * B, Vl), local.contiguous(), group=self.group)
        COMM.record("all_gather", local.numel() * local.element_size())
        V = full.shape[1]
        full.copy_(buf.permute(1, 0, 2).reshape(B, W * Vl)[:, :V])
        return full

    def all_gather_flat(self, local: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """Contiguous ``local`` of every rank -> ``out`` = [W * local.numel()] in rank order."""
        dist.all_gather_into_tensor(out, local.contiguous(), group=self.group)
        COMM.record("all_gather", local.numel() * local.element_size())
        return out

    def broadcast_obj(self, obj, src: int = 0):
        lst = [obj]
        dist.broadcast_object_list(lst, src=src, group=self.group)
        return lst[0]


def init_from_env(backend: str = "nccl") -> TPGroup | None:
    """Initialise torch.distributed from torchrun's env; None when WORLD_SIZE is 1."""
    import os
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if ws <= 1:
        return None
    if not dist.is_initialized():
        if backend == "nccl":
            torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        from datetime import timedelta
        # a lost rank ends the others' next collective with an error instead of a long hang
        timeout = timedelta(seconds=float(os.environ.get("AIR_PG_TIMEOUT_S", "300")))
        dist.init_process_group(backend=backend, timeout=timeout)
    return TPGroup()
