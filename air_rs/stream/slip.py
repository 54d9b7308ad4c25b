"""S.L.I.P. layer streaming: run a model whose layers do not stay in HBM (reference
``src/slip.rs`` SlipDispatcher streaming mode and ``src/weight_streamer.rs`` load_layer /
prefetch_layer).

The per-layer weights live in pinned host memory, already in the kernels' device layouts
(tiled Q4_K, split Q8_0), so a layer is a handful of plain host->device copies. ``n_slots``
device slots (double buffering by default) hold the layers in flight: while the compute
stream runs layer i from slot i % n, a copy stream fills the next slot with layer i+1; the
copy into a slot waits on an event recorded after the last kernel that read it. Per-layer
copy and compute intervals are timed with CUDA events on their own streams, which gives the
overlap ratio.

Reference (storage side): the reference memory-maps the GGUF file and dequantises each
layer into fresh device tensors on every forward; NVMe -> page cache -> pinned is here the
load step (``LlamaWeights(layer_device="cpu")``) and the per-step stream is pinned -> HBM.
"""
from __future__ import annotations

import copy
import dataclasses
from dataclasses import dataclass, field

import torch

from .. import ops
from ..models.llama import LayerWeights, layer_tensors


def _device_clone(lw: LayerWeights, device) -> LayerWeights:
    """An empty device-resident LayerWeights with the same shapes (a slot)."""
    out = copy.copy(lw)
    for f in dataclasses.fields(lw):
        v = getattr(lw, f.name)
        if isinstance(v, torch.Tensor):
            setattr(out, f.name, torch.empty_like(v, device=device))
        elif isinstance(v, ops.QWeight):
            setattr(out, f.name, _qw_empty(v, device))
        elif isinstance(v, list) and v and isinstance(v[0], ops.QWeight):
            setattr(out, f.name, [_qw_empty(q, device) for q in v])
    return out


def _qw_empty(q: ops.QWeight, device) -> ops.QWeight:
    return ops.QWeight(q.fmt, torch.empty_like(q.data, device=device),
                       None if q.scales is None else torch.empty_like(q.scales, device=device),
                       q.N, q.K, q.qtype, q.parts)


@dataclass
class StreamStats:
    layers_loaded: int = 0
    bytes_h2d: int = 0
    copy_ms: float = 0.0
    compute_ms: float = 0.0
    underruns: int = 0           # layers whose compute waited for their copy
    stall_ms: float = 0.0        # compute-stream idle time spent waiting on copies
    _pending: list = field(default_factory=list)
    _last_end: object = None

    def overlap_ratio(self, step_ms: float) -> float:
        """Fraction of the shorter of (copy, compute) hidden under the other."""
        lo = min(self.copy_ms, self.compute_ms)
        if lo <= 0:
            return 0.0
        return max(0.0, min(1.0, (self.copy_ms + self.compute_ms - step_ms) / lo))


class LayerStreamer:
    def __init__(self, host_layers: list[LayerWeights], device, n_slots: int = 2, timing: bool = True,
                 resident=()):
        """``resident``: layer indices copied to the device once and kept there (partial
        residency); the other layers cycle through the ``n_slots`` streaming slots."""
        if n_slots < 2:
            raise ValueError("layer streaming needs at least two device slots")
        self.host = host_layers
        self.device = torch.device(device)
        self.n = n_slots
        self.resident: dict[int, LayerWeights] = {}
        for li in sorted(set(resident)):
            lw = _device_clone(host_layers[li], self.device)
            for dst, src in zip(layer_tensors(lw), layer_tensors(host_layers[li])):
                dst.copy_(src)
            self.resident[li] = lw
        self.streamed = [li for li in range(len(host_layers)) if li not in self.resident]
        self._pos = {li: i for i, li in enumerate(self.streamed)}
        self._deferred: int | None = None
        self.slots = [_device_clone(host_layers[0], self.device) for _ in range(n_slots)]
        self.slot_tensors = [layer_tensors(s) for s in self.slots]
        self.copy_stream = torch.cuda.Stream(self.device)
        self.loaded = [-1] * n_slots
        self.ready: list[torch.cuda.Event | None] = [None] * n_slots
        self.free: list[torch.cuda.Event | None] = [None] * n_slots
        self.timing = timing
        self.stats = StreamStats()
        self._compute_start: dict[int, torch.cuda.Event] = {}

    def _slot(self, li: int) -> int:
        return self._pos[li] % self.n

    def _next_streamed(self, li: int) -> int:
        """The first streamed layer after li (wrapping to the next step)."""
        for d in range(1, len(self.host) + 1):
            nxt = (li + d) % len(self.host)
            if nxt not in self.resident:
                return nxt
        return -1

    def prefetch(self, li: int):
        """Issue the host->device copy of layer li into its slot (no-op if already there)."""
        if li < 0 or li >= len(self.host) or li in self.resident:
            return
        s = self._slot(li)
        if self.loaded[s] == li:
            return
        with torch.cuda.stream(self.copy_stream):
            if self.free[s] is not None:
                self.copy_stream.wait_event(self.free[s])
            t0 = torch.cuda.Event(enable_timing=True) if self.timing else None
            if t0 is not None:
                t0.record()
            nb = 0
            for dst, src in zip(self.slot_tensors[s], layer_tensors(self.host[li])):
                dst.copy_(src, non_blocking=True)
                nb += src.numel() * src.element_size()
            ev = torch.cuda.Event(enable_timing=self.timing)
            ev.record()
        self.ready[s] = ev
        self.loaded[s] = li
        self.stats.layers_loaded += 1
        self.stats.bytes_h2d += nb
        if t0 is not None:
            self.stats._pending.append(("copy", t0, ev))

    def get(self, li: int) -> LayerWeights:
        """Layer li on the device for the compute stream; starts fetching the next streamed
        layer."""
        if li in self.resident:
            self.prefetch(self._next_streamed(li))
            return self.resident[li]
        self.prefetch(li)
        s = self._slot(li)
        cs = torch.cuda.current_stream(self.device)
        cs.wait_event(self.ready[s])
        # the next streamed layer's slot is free once the layer that used it last is done;
        # after the last layer this starts the first streamed layer of the next step. When the
        # next layer maps to this very slot (an odd number of streamed layers wrapping around),
        # its copy has to wait for this layer's release.
        nxt = self._next_streamed(li)
        if nxt >= 0 and self._slot(nxt) == s and nxt != li:
            self._deferred = nxt
        else:
            self.prefetch(nxt)
        if self.timing:
            e = torch.cuda.Event(enable_timing=True)
            e.record(cs)
            self._compute_start[li] = e
        return self.slots[s]

    def release(self, li: int):
        """Record that the compute stream has enqueued every kernel reading layer li."""
        if li in self.resident:
            return
        s = self._slot(li)
        ev = torch.cuda.Event(enable_timing=self.timing)
        ev.record(torch.cuda.current_stream(self.device))
        self.free[s] = ev
        if self._deferred is not None:
            nxt, self._deferred = self._deferred, None
            self.prefetch(nxt)
        st = self._compute_start.pop(li, None)
        if st is not None:
            # the first layer of a step follows host work (sampling, scheduling): no gap check
            self.stats._pending.append(("compute0" if li == 0 else "compute", st, ev))

    UNDERRUN_MS = 0.02

    def collect(self):
        """Fold finished event pairs into the copy / compute totals (synchronises them). A gap
        between one layer's compute end and the next layer's compute start is time the compute
        stream spent waiting for a copy (a slot underrun)."""
        st = self.stats
        for kind, a, b in st._pending:
            b.synchronize()
            ms = a.elapsed_time(b)
            if kind == "copy":
                st.copy_ms += ms
            else:
                st.compute_ms += ms
                if kind == "compute" and st._last_end is not None:
                    gap = st._last_end.elapsed_time(a)
                    if gap > self.UNDERRUN_MS:
                        st.underruns += 1
                        st.stall_ms += gap
                st._last_end = b
        st._pending.clear()
        return st
