"""KV host tier: swap a sequence's paged KV blocks between HBM and pinned host memory
(reference ``src/kv_swap.rs``: KvSwapManager evict / restore / maybe_evict over the paged
bookkeeping, with caller-supplied GPU read/write callbacks that nothing wires up).

Here eviction gathers the sequence's blocks of every layer from the HBM pool
(``kv[L, num_blocks, 2, n_kv, block, d]``) into one pinned host buffer with a single
device->host copy on a side stream, then returns the blocks to the allocator; restore
allocates fresh blocks, copies host->device on the side stream and scatters them into the
pool. The compute stream waits on the side stream's event before it touches the pool again.
Used by the engine to preempt sequences when the pool runs out of blocks.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class _Evicted:
    host: torch.Tensor          # [L, n_blocks, 2, n_kv, block, d] pinned
    n_blocks: int
    event: torch.cuda.Event | None


class KvSwapManager:
    def __init__(self, kv: torch.Tensor, seqs, stream: torch.cuda.Stream | None = None):
        self.kv = kv
        self.seqs = seqs
        self.stream = stream if stream is not None else (torch.cuda.Stream(kv.device) if kv.is_cuda else None)
        self._store: dict[int, _Evicted] = {}
        self.bytes_out = 0
        self.bytes_in = 0

    def _run(self, fn):
        if self.stream is None:
            return fn()
        self.stream.wait_stream(torch.cuda.current_stream(self.kv.device))
        with torch.cuda.stream(self.stream):
            return fn()

    def evict(self, seq: int) -> list[int]:
        """Copy ``seq``'s blocks to host and release them; returns the freed block ids."""
        if seq in self._store:
            raise RuntimeError(f"sequence {seq} is already evicted")
        blocks = self.seqs.block_table(seq)
        n = len(blocks)
        host = torch.empty((self.kv.shape[0], n) + tuple(self.kv.shape[2:]), dtype=self.kv.dtype,
                           pin_memory=self.kv.is_cuda)
        idx = torch.tensor(blocks, dtype=torch.long, device=self.kv.device)

        def go():
            host.copy_(self.kv.index_select(1, idx), non_blocking=True)
            if self.kv.is_cuda:
                ev = torch.cuda.Event()
                ev.record()
                return ev
            return None
        ev = self._run(go)
        # the blocks may be reallocated only once the copy has read them
        if ev is not None:
            torch.cuda.current_stream(self.kv.device).wait_event(ev)
        self.seqs.swap_out(seq)
        self._store[seq] = _Evicted(host, n, ev)
        self.bytes_out += host.numel() * host.element_size()
        return blocks

    def restore(self, seq: int) -> list[int]:
        """Re-acquire device blocks for ``seq`` and copy its KV back; returns the new ids."""
        ent = self._store.pop(seq)
        blocks = self.seqs.swap_in(seq)
        idx = torch.tensor(blocks, dtype=torch.long, device=self.kv.device)

        def go():
            if ent.event is not None:
                torch.cuda.current_stream().wait_event(ent.event)
            dev = ent.host.to(self.kv.device, non_blocking=True)
            self.kv.index_copy_(1, idx, dev)
            if self.kv.is_cuda:
                ev = torch.cuda.Event()
                ev.record()
                return ev
            return None
        ev = self._run(go)
        if ev is not None:
            torch.cuda.current_stream(self.kv.device).wait_event(ev)
        self.bytes_in += ent.host.numel() * ent.host.element_size()
        return blocks

    def is_evicted(self, seq: int) -> bool:
        return seq in self._store

    def evicted_count(self) -> int:
        return len(self._store)

    def maybe_evict(self, seq: int, free_threshold: int) -> bool:
        """Evict ``seq`` if the pool has fewer than ``free_threshold`` free blocks."""
        if self.seqs.allocator.num_free_blocks() >= free_threshold or seq in self._store:
            return False
        self.evict(seq)
        return True

    def drop(self, seq: int):
        """Forget an evicted sequence (its request was aborted)."""
        self._store.pop(seq, None)
