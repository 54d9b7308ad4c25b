"""Data-parallel replicas behind one endpoint (the reference names the strategy,
``ShardStrategy::Replicated`` in ``src/distributed.rs:229-238``, without a router).

``ReplicaRouter`` is a ``Dispatcher`` over several independent dispatchers, typically one
``EngineDispatcher`` per GPU each holding a full copy of the model (``serve --dp N``). Each
request goes to the replica with the fewest requests in flight (ties: round robin), and
the whole stream stays on that replica. A replica whose generate raises before its first
chunk is skipped for that request and the next-least-loaded one is tried, so one failed
GPU does not fail the endpoint. Embeddings are routed the same way."""
from __future__ import annotations

import itertools
import threading

from .dispatcher import Dispatcher, FinishReason, TokenChunk


class ReplicaRouter(Dispatcher):
    def __init__(self, replicas: list[Dispatcher], model_name: str | None = None):
        if not replicas:
            raise ValueError("ReplicaRouter needs at least one replica")
        self.replicas = list(replicas)
        self.model_name = model_name
        self.in_flight = [0] * len(replicas)
        self.served = [0] * len(replicas)
        self._rr = itertools.count()
        self._lock = threading.Lock()

    def list_models(self):
        return [self.model_name] if self.model_name else self.replicas[0].list_models()

    def count_tokens(self, text: str) -> int:
        return self.replicas[0].count_tokens(text)

    def _order(self) -> list[int]:
        with self._lock:
            start = next(self._rr) % len(self.replicas)
            idx = list(range(start, len(self.replicas))) + list(range(start))
            return sorted(idx, key=lambda i: self.in_flight[i])      # stable: round robin on ties

    async def generate(self, config):
        last_err = None
        for i in self._order():
            with self._lock:
                self.in_flight[i] += 1
            started = False
            try:
                async for chunk in self.replicas[i].generate(config):
                    started = True
                    yield chunk
                with self._lock:
                    self.served[i] += 1
                return
            except Exception as e:      # a replica that fails before streaming: try the next
                if started:
                    yield TokenChunk(finish_reason=FinishReason.ERROR, error=str(e))
                    return
                last_err = e
            finally:
                with self._lock:
                    self.in_flight[i] -= 1
        yield TokenChunk(finish_reason=FinishReason.ERROR, error=f"all replicas failed: {last_err}")

    def embed(self, text: str) -> list[float]:
        last_err = None
        for i in self._order():
            try:
                return self.replicas[i].embed(text)
            except Exception as e:
                last_err = e
        raise RuntimeError(f"all replicas failed: {last_err}")

    def shutdown(self):
        for r in self.replicas:
            if hasattr(r, "shutdown"):
                r.shutdown()
