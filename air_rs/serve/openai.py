"""OpenAI-compatible schema helpers, API keys, rate limiting, latency histograms and the
Prometheus exposition (reference ``src/openai_api.rs`` and ``src/api.rs:252-345``; there
these were library code not mounted on the router, here the server uses them).
"""
from __future__ import annotations

import hashlib
import hmac
import math
import threading
import time
import uuid
from dataclasses import dataclass, field


class ApiErrorCode:
    INVALID_REQUEST = ("invalid_request_error", 400)
    AUTHENTICATION = ("authentication_error", 401)
    MODEL_NOT_FOUND = ("model_not_found", 404)
    RATE_LIMIT = ("rate_limit_exceeded", 429)
    SERVER_ERROR = ("server_error", 500)


class ApiError(Exception):
    """``{"error": {"message", "type", "code"}}`` envelope with its HTTP status."""

    def __init__(self, message: str, kind=ApiErrorCode.INVALID_REQUEST, code: str | None = None):
        super().__init__(message)
        self.message = message
        self.type, self.status = kind
        self.code = code

    def body(self) -> dict:
        return {"error": {"message": self.message, "type": self.type, "code": self.code}}

    @classmethod
    def model_not_found(cls, model: str) -> "ApiError":
        return cls(f"The model '{model}' does not exist", ApiErrorCode.MODEL_NOT_FOUND, "model_not_found")


def new_id(prefix: str) -> str:
    return f"{prefix}-{uuid.uuid4().hex[:24]}"


def now() -> int:
    return int(time.time())


def validate_sampling(req: dict):
    t = req.get("temperature")
    if t is not None and not (0.0 <= float(t) <= 2.0):
        raise ApiError("temperature must be between 0 and 2")
    p = req.get("top_p")
    if p is not None and not (0.0 < float(p) <= 1.0):
        raise ApiError("top_p must be in (0, 1]")
    mt = req.get("max_tokens", req.get("max_output_tokens"))
    if mt is not None and int(mt) < 1:
        raise ApiError("max_tokens must be >= 1")


def stop_list(stop) -> list[str]:
    if stop is None:
        return []
    if isinstance(stop, str):
        return [stop]
    if isinstance(stop, list) and all(isinstance(s, str) for s in stop):
        return stop
    raise ApiError("stop must be a string or a list of strings")


def usage(prompt_tokens: int, completion_tokens: int) -> dict:
    return {"prompt_tokens": prompt_tokens, "completion_tokens": completion_tokens,
            "total_tokens": prompt_tokens + completion_tokens}


def chat_chunk(cid: str, model: str, delta: dict, finish_reason: str | None = None) -> dict:
    return {"id": cid, "object": "chat.completion.chunk", "created": now(), "model": model,
            "choices": [{"index": 0, "delta": delta, "finish_reason": finish_reason}]}


def to_sse(obj) -> str:
    import json
    return f"data: {json.dumps(obj)}\n\n"


class ApiKeyStore:
    """API keys kept as SHA-256 digests, compared in constant time."""

    def __init__(self, keys: list[str] | None = None):
        self._digests = {hashlib.sha256(k.encode()).hexdigest() for k in (keys or [])}

    def add(self, key: str):
        self._digests.add(hashlib.sha256(key.encode()).hexdigest())

    @property
    def enabled(self) -> bool:
        return bool(self._digests)

    def check(self, authorization: str | None) -> bool:
        if not self.enabled:
            return True
        if not authorization or not authorization.startswith("Bearer "):
            return False
        d = hashlib.sha256(authorization[7:].strip().encode()).hexdigest()
        return any(hmac.compare_digest(d, x) for x in self._digests)


class RateLimiter:
    """Token bucket per client key: ``rate`` requests/s with ``burst`` capacity."""

    def __init__(self, rate: float, burst: int):
        self.rate, self.burst = rate, burst
        self._buckets: dict[str, tuple[float, float]] = {}
        self._lock = threading.Lock()

    def allow(self, key: str, now_s: float | None = None) -> bool:
        t = time.monotonic() if now_s is None else now_s
        with self._lock:
            tokens, last = self._buckets.get(key, (float(self.burst), t))
            tokens = min(self.burst, tokens + (t - last) * self.rate)
            ok = tokens >= 1.0
            self._buckets[key] = (tokens - 1.0 if ok else tokens, t)
            return ok


class LatencyHistogram:
    BUCKETS_MS = (5, 10, 25, 50, 100, 250, 500, 1000, 2500, 5000, 10000, 30000)

    def __init__(self):
        self.samples: list[float] = []
        self.counts = [0] * (len(self.BUCKETS_MS) + 1)
        self.total = 0.0
        self._lock = threading.Lock()

    def record(self, ms: float):
        with self._lock:
            self.samples.append(ms)
            if len(self.samples) > 10000:
                self.samples = self.samples[-5000:]
            self.total += ms
            for i, b in enumerate(self.BUCKETS_MS):
                if ms <= b:
                    self.counts[i] += 1
                    break
            else:
                self.counts[-1] += 1

    def percentile(self, p: float) -> float:
        with self._lock:
            if not self.samples:
                return 0.0
            s = sorted(self.samples)
            k = max(0, min(len(s) - 1, math.ceil(p / 100 * len(s)) - 1))
            return s[k]

    @property
    def count(self) -> int:
        return sum(self.counts)


@dataclass
class PrometheusMetrics:
    requests_total: int = 0
    requests_failed: int = 0
    tokens_generated: int = 0
    prompt_tokens: int = 0
    active_requests: int = 0
    ttft: LatencyHistogram = field(default_factory=LatencyHistogram)
    latency: LatencyHistogram = field(default_factory=LatencyHistogram)
    start_time: float = field(default_factory=time.time)

    def render(self, model: str = "air-rs", gauges: dict | None = None) -> str:
        """Prometheus text; ``gauges`` (engine statistics) are exported as ``air_<name>``."""
        lines = []

        def metric(name, kind, help_, value):
            lines.append(f"# HELP {name} {help_}")
            lines.append(f"# TYPE {name} {kind}")
            lines.append(f'{name}{{model="{model}"}} {value}')

        metric("air_requests_total", "counter", "Requests served", self.requests_total)
        metric("air_requests_failed_total", "counter", "Requests that failed", self.requests_failed)
        metric("air_tokens_generated_total", "counter", "Completion tokens generated", self.tokens_generated)
        metric("air_prompt_tokens_total", "counter", "Prompt tokens processed", self.prompt_tokens)
        metric("air_active_requests", "gauge", "Requests in flight", self.active_requests)
        metric("air_uptime_seconds", "gauge", "Server uptime", int(time.time() - self.start_time))
        for hname, h in (("air_ttft_ms", self.ttft), ("air_request_latency_ms", self.latency)):
            lines.append(f"# HELP {hname} Latency histogram (ms)")
            lines.append(f"# TYPE {hname} histogram")
            cum = 0
            for b, c in zip(h.BUCKETS_MS, h.counts):
                cum += c
                lines.append(f'{hname}_bucket{{model="{model}",le="{b}"}} {cum}')
            lines.append(f'{hname}_bucket{{model="{model}",le="+Inf"}} {h.count}')
            lines.append(f'{hname}_sum{{model="{model}"}} {h.total:.3f}')
            lines.append(f'{hname}_count{{model="{model}"}} {h.count}')
            for q in (50, 95, 99):
                lines.append(f'{hname}_p{q}{{model="{model}"}} {h.percentile(q):.3f}')
        for k, v in sorted((gauges or {}).items()):
            if isinstance(v, (int, float)) and not isinstance(v, bool):
                metric(f"air_{k}", "gauge", f"engine {k.replace('_', ' ')}", v)
        return "\n".join(lines) + "\n"
