"""Tracing: NVTX ranges around engine phases and layers, host span records, and
``torch.profiler`` traces on demand.

The reference lists ``tracing`` as a dependency but emits no spans; its profiling is
wall-clock ``Instant`` timers (``src/metrics.rs:20-199`` InferenceMetrics / LayerTiming).
Here ``AIR_TRACE=1`` (or ``enable()``) turns on:

* NVTX ranges (``torch.cuda.nvtx``) named ``air/<phase>`` — visible in Nsight Systems and in
  ``ncu --nvtx`` filters; ranges opened while a CUDA graph is captured are host-side only;
* a host span list (name, start ns, duration ns, depth) kept in memory, exportable as a
  Chrome trace JSON (``dump_chrome``), which also works without a GPU.

``profile(path)`` wraps a region in ``torch.profiler`` (CPU + CUDA activities) and writes a
Chrome trace. With tracing off, ``span`` costs one attribute read.
"""
from __future__ import annotations

import contextlib
import json
import os
import threading
import time
from dataclasses import dataclass

_state = threading.local()
_enabled = os.environ.get("AIR_TRACE", "0").lower() in ("1", "true", "yes", "on")
_spans: list["Span"] = []
_lock = threading.Lock()
_MAX_SPANS = 1_000_000


@dataclass
class Span:
    name: str
    start_ns: int
    dur_ns: int
    depth: int
    tid: int


def enabled() -> bool:
    return _enabled


def enable(on: bool = True):
    global _enabled
    _enabled = bool(on)


def clear():
    with _lock:
        _spans.clear()


def spans() -> list[Span]:
    with _lock:
        return list(_spans)


def _nvtx():
    try:
        import torch
        if torch.cuda.is_available():
            return torch.cuda.nvtx
    except Exception:
        pass
    return None


@contextlib.contextmanager
def span(name: str):
    """NVTX range + host span ``air/<name>`` while tracing is on; nothing otherwise."""
    if not _enabled:
        yield
        return
    nv = _nvtx()
    depth = getattr(_state, "depth", 0)
    _state.depth = depth + 1
    if nv is not None:
        nv.range_push("air/" + name)
    t0 = time.perf_counter_ns()
    try:
        yield
    finally:
        dt = time.perf_counter_ns() - t0
        if nv is not None:
            nv.range_pop()
        _state.depth = depth
        with _lock:
            if len(_spans) < _MAX_SPANS:
                _spans.append(Span(name, t0, dt, depth, threading.get_ident()))


def traced(name: str | None = None):
    """Decorator form of ``span``."""
    def deco(fn):
        label = name or fn.__qualname__

        def wrapper(*a, **kw):
            if not _enabled:
                return fn(*a, **kw)
            with span(label):
                return fn(*a, **kw)
        wrapper.__wrapped__ = fn
        wrapper.__name__ = fn.__name__
        wrapper.__doc__ = fn.__doc__
        return wrapper
    return deco


def summary() -> dict[str, dict]:
    """Per-name count / total / mean milliseconds of the recorded host spans."""
    out: dict[str, dict] = {}
    for s in spans():
        d = out.setdefault(s.name, {"count": 0, "total_ms": 0.0})
        d["count"] += 1
        d["total_ms"] += s.dur_ns / 1e6
    for d in out.values():
        d["mean_ms"] = d["total_ms"] / d["count"]
    return out


def dump_chrome(path: str):
    """Write the host spans as a Chrome trace (``chrome://tracing`` / Perfetto)."""
    ev = [{"name": s.name, "ph": "X", "ts": s.start_ns / 1e3, "dur": s.dur_ns / 1e3,
           "pid": os.getpid(), "tid": s.tid, "args": {"depth": s.depth}} for s in spans()]
    with open(path, "w") as f:
        json.dump({"traceEvents": ev, "displayTimeUnit": "ms"}, f)
    return path


@contextlib.contextmanager
def profile(path: str, cuda: bool | None = None):
    """``torch.profiler`` over the block, exported as a Chrome trace to ``path``."""
    import torch
    from torch.profiler import ProfilerActivity
    acts = [ProfilerActivity.CPU]
    if cuda is None:
        cuda = torch.cuda.is_available()
    if cuda:
        acts.append(ProfilerActivity.CUDA)
    with torch.profiler.profile(activities=acts, record_shapes=False) as prof:
        yield prof
    prof.export_chrome_trace(path)
