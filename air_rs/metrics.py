"""Inference metrics (same summary fields as the reference's ``src/metrics.rs:40-199``),
plus device-timed step latencies recorded with CUDA events."""
from __future__ import annotations

import time
from dataclasses import dataclass, field


@dataclass
class LayerTiming:
    layer_id: int
    io_ms: float = 0.0
    compute_ms: float = 0.0


@dataclass
class InferenceMetrics:
    start_time: float = field(default_factory=time.perf_counter)
    first_token_time: float | None = None
    tokens_generated: int = 0
    prompt_tokens: int = 0
    layer_timings: list[LayerTiming] = field(default_factory=list)
    device_step_ms: list[float] = field(default_factory=list)

    def start(self):
        self.start_time = time.perf_counter()
        self.first_token_time = None
        self.tokens_generated = 0
        self.layer_timings.clear()
        self.device_step_ms.clear()

    def mark_first_token(self):
        if self.first_token_time is None:
            self.first_token_time = time.perf_counter()

    def record_token(self):
        self.tokens_generated += 1

    def record_layer(self, layer_id: int, io_ms: float, compute_ms: float):
        self.layer_timings.append(LayerTiming(layer_id, io_ms, compute_ms))

    def ttft_ms(self) -> float:
        if self.first_token_time is None:
            return 0.0
        return (self.first_token_time - self.start_time) * 1e3

    def total_ms(self) -> float:
        return (time.perf_counter() - self.start_time) * 1e3

    def tokens_per_second(self) -> float:
        """Decode rate after the first token (the reference's tok/s excludes prefill here)."""
        if self.first_token_time is None or self.tokens_generated <= 1:
            return 0.0
        dt = time.perf_counter() - self.first_token_time
        return (self.tokens_generated - 1) / dt if dt > 0 else 0.0

    def pipeline_efficiency(self) -> float:
        io = sum(t.io_ms for t in self.layer_timings)
        comp = sum(t.compute_ms for t in self.layer_timings)
        tot = max(io, comp) if self.layer_timings else 0.0
        return comp / tot if tot > 0 else 0.0

    def summary(self) -> str:
        return (f"TTFT {self.ttft_ms():.1f} ms | {self.tokens_generated} tokens | "
                f"{self.tokens_per_second():.1f} tok/s | total {self.total_ms():.1f} ms")
