"""Expert VRAM scheduler: MoE experts kept in pinned host memory, with an LRU set of them
resident in device slots (reference ``src/moe.rs:345-504`` ExpertVramScheduler:
ensure_resident / get / evict_lru / hit_rate / prefetch_hints).

``ExpertVramScheduler`` is the bookkeeping: a capacity, an LRU order, hit / load / eviction
counters and per-expert use counts; the payload of a resident entry is whatever the caller's
``load_fn`` returns.

``DeviceExpertCache`` puts it on the GPU: ``capacity`` slots, each holding one expert's fused
gate|up and down weights in the kernels' device layouts. The MoE layer routes on the device,
reads back which experts any token picked (one small device->host copy per MoE layer), makes
those resident — a miss is two host->device copies into the slot of the least recently used
expert, issued on the compute stream after the kernels that last read that slot — and runs
only the picked experts. Steps that route through the cache read routing on the host, so they
run without CUDA graphs.
"""
from __future__ import annotations

from collections import OrderedDict
from typing import Callable, Hashable

import torch


class ExpertVramScheduler:
    def __init__(self, capacity: int):
        if capacity < 1:
            raise ValueError("expert VRAM capacity must be >= 1")
        self.capacity = capacity
        self._res: OrderedDict[Hashable, object] = OrderedDict()   # last item = most recent
        self.usage_freq: dict[Hashable, int] = {}
        self.eviction_count = 0
        self.load_count = 0
        self.hit_count = 0

    def ensure_resident(self, needed, load_fn: Callable, evict_fn: Callable | None = None):
        """Make every id in ``needed`` resident (``load_fn(id, evicted_payload_or_None)`` on a
        miss). Ids in ``needed`` are never evicted by this call; more than ``capacity`` of them
        raises."""
        needed = list(dict.fromkeys(needed))
        if len(needed) > self.capacity:
            raise RuntimeError(f"{len(needed)} experts needed at once, capacity {self.capacity}")
        keep = set(needed)
        for eid in needed:
            if eid in self._res:
                self.hit_count += 1
                self._res.move_to_end(eid)
            else:
                freed = None
                if len(self._res) >= self.capacity:
                    freed = self._evict_lru(keep, evict_fn)
                try:
                    payload = load_fn(eid, freed)
                except Exception as e:
                    raise RuntimeError(f"failed to load expert {eid}: {e}") from e
                self._res[eid] = payload
                self.load_count += 1
            self.usage_freq[eid] = self.usage_freq.get(eid, 0) + 1

    def _evict_lru(self, keep, evict_fn):
        for eid in self._res:
            if eid not in keep:
                payload = self._res.pop(eid)
                self.eviction_count += 1
                if evict_fn is not None:
                    evict_fn(eid, payload)
                return payload
        raise RuntimeError("no evictable expert")

    def get(self, eid):
        try:
            return self._res[eid]
        except KeyError:
            raise KeyError(f"expert {eid} not resident; call ensure_resident first") from None

    def is_resident(self, eid) -> bool:
        return eid in self._res

    def resident_count(self) -> int:
        return len(self._res)

    def hit_rate(self) -> float:
        t = self.hit_count + self.load_count
        return 1.0 if t == 0 else self.hit_count / t

    def prefetch_hints(self, n: int) -> list:
        """The ``n`` most used experts that are not resident, most used first."""
        cand = [(f, eid) for eid, f in self.usage_freq.items() if eid not in self._res]
        cand.sort(key=lambda x: -x[0])
        return [eid for _, eid in cand[:n]]

    def reset_stats(self):
        self.eviction_count = self.load_count = self.hit_count = 0


class DeviceExpertCache:
    """Device slots for host-resident experts of every MoE layer of a runner."""

    def __init__(self, layers, capacity: int, device):
        from .. import ops
        self.device = torch.device(device)
        self.layers = layers
        self.layer_index = {id(lw): i for i, lw in enumerate(layers)}
        per_layer = max(len(lw.experts_gu) for lw in layers)
        self.sched = ExpertVramScheduler(capacity)
        g0, d0 = layers[0].experts_gu[0], layers[0].experts_down[0]

        def empty(q):
            return ops.QWeight(q.fmt, torch.empty_like(q.data, device=self.device),
                               None if q.scales is None else torch.empty_like(q.scales, device=self.device),
                               q.N, q.K, q.qtype, q.parts)
        self.slots = [(empty(g0), empty(d0)) for _ in range(capacity)]
        self._free = list(range(capacity))[::-1]
        self.per_layer = per_layer
        self.bytes_h2d = 0

    def _load(self, key, freed):
        li, j = key
        slot = freed if freed is not None else self._free.pop()
        gu_d, dn_d = self.slots[slot]
        lw = self.layers[li]
        for dst, src in ((gu_d, lw.experts_gu[j]), (dn_d, lw.experts_down[j])):
            dst.data.copy_(src.data, non_blocking=True)
            self.bytes_h2d += src.data.numel() * src.data.element_size()
            if src.scales is not None:
                dst.scales.copy_(src.scales, non_blocking=True)
                self.bytes_h2d += src.scales.numel() * src.scales.element_size()
        return slot

    def experts_for(self, lw, picked: torch.Tensor):
        """``picked``: bool [E] (any token routed to expert e). Yields (gu, down, e) device
        weights of this rank's picked experts, at most ``capacity`` resident at a time; a slot
        reused within one layer is refilled in stream order after its last reader."""
        li = self.layer_index[id(lw)]
        ids = lw.expert_ids or list(range(len(lw.experts_gu)))
        sel = picked.tolist()
        local = [j for j, e in enumerate(ids) if sel[e]]
        # resident experts first, so a chunk does not evict one that a later chunk needs
        local.sort(key=lambda j: not self.sched.is_resident((li, j)))
        cap = self.sched.capacity
        for c in range(0, len(local), cap):
            chunk = local[c:c + cap]
            keys = [(li, j) for j in chunk]
            self.sched.ensure_resident(keys, self._load)
            for j, k in zip(chunk, keys):
                gu_d, dn_d = self.slots[self.sched.get(k)]
                yield gu_d, dn_d, ids[j]

    def stats(self) -> dict:
        s = self.sched
        return {"capacity": s.capacity, "resident": s.resident_count(), "hits": s.hit_count,
                "loads": s.load_count, "evictions": s.eviction_count, "hit_rate": s.hit_rate(),
                "bytes_h2d": self.bytes_h2d}
