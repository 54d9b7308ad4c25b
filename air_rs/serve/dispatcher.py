"""Dispatcher seam between the HTTP layer and the engine (reference ``src/dispatcher.rs``).

``Dispatcher.generate(config)`` yields ``TokenChunk`` items (a token's text, then one final
stop chunk with a finish reason); ``list_models()`` names the served models.

``EngineDispatcher`` owns a core ``Engine`` on one background thread that runs the
continuous-batching loop: requests from any number of HTTP handlers are admitted into the
running batch (the reference serves one request at a time from a single task,
``src/scheduler.rs:36-100``, and its stream stops after 32 tokens because generation runs
to completion before the bounded channel is drained, ``src/inference_step.rs:193,361``).
Per-request ``temperature`` / ``top_p`` / ``stop`` / grammar are honoured.
"""
from __future__ import annotations

import asyncio
import itertools
import queue
import threading
import time
from dataclasses import dataclass, field
from typing import AsyncIterator

from ..runtime.engine import SamplingParams
from ..structured.text import StopChecker


class FinishReason:
    STOP = "stop"
    LENGTH = "length"
    ERROR = "error"
    ABORT = "abort"


@dataclass
class TokenChunk:
    text: str = ""
    token_id: int = -1
    finish_reason: str | None = None     # set on the final chunk only
    error: str | None = None

    @property
    def is_stop(self) -> bool:
        return self.finish_reason is not None


@dataclass
class GenerateConfig:
    """Dispatcher-level request (defaults from ``src/dispatcher.rs:82-121``)."""
    model: str = ""
    prompt: str = ""
    prompt_ids: list[int] | None = None
    max_tokens: int = 256
    temperature: float = 0.8
    top_p: float = 0.95
    top_k: int = 40
    repetition_penalty: float = 1.1
    stop: list[str] = field(default_factory=list)
    draft_model: str | None = None
    gbnf: str | None = None
    json_mode: bool = False


class Dispatcher:
    async def generate(self, config: GenerateConfig) -> AsyncIterator[TokenChunk]:  # pragma: no cover
        raise NotImplementedError
        yield

    def list_models(self) -> list[str]:  # pragma: no cover
        raise NotImplementedError

    def count_tokens(self, text: str) -> int:
        return max(1, len(text) // 4)

    def embed(self, text: str) -> list[float]:  # pragma: no cover
        raise NotImplementedError


class MockDispatcher(Dispatcher):
    """Deterministic echo dispatcher for tests (reference ``MockDispatcher``)."""

    def __init__(self, model: str = "mock", tokens: list[str] | None = None):
        self.model = model
        self.tokens = tokens or ["Hello", ",", " world", "!"]

    async def generate(self, config):
        n = 0
        for t in self.tokens:
            if n >= config.max_tokens:
                yield TokenChunk(finish_reason=FinishReason.LENGTH)
                return
            n += 1
            yield TokenChunk(t, n)
            await asyncio.sleep(0)
        yield TokenChunk(finish_reason=FinishReason.STOP)

    def list_models(self):
        return [self.model]

    def embed(self, text):
        return [float(len(text)), 0.0, 1.0]


class EngineDispatcher(Dispatcher):
    """Continuous-batching engine loop on a worker thread."""

    def __init__(self, engine, model_name: str = "air-rs", health=None):
        """``health``: an ``air_rs.parallel.health.Heartbeat`` checked before every step."""
        self.engine = engine               # air_rs.runtime.engine.Engine
        self.model_name = model_name
        self.health = health
        self.errors = 0
        self._submit: queue.Queue = queue.Queue()
        self._texts: list[str] | None = None
        self._lock = threading.Lock()
        self._stop = threading.Event()
        self._ids = itertools.count()
        self.requests_served = 0
        self._thread = threading.Thread(target=self._loop, name="air_rs_engine", daemon=True)
        self._thread.start()

    def list_models(self):
        return [self.model_name]

    def count_tokens(self, text: str) -> int:
        return len(self.engine.tokenizer.encode(text))

    def shutdown(self):
        self._stop.set()
        self._submit.put(None)
        self._thread.join(timeout=5)

    # -- engine thread ------------------------------------------------------------
    def _loop(self):
        eng = self.engine
        while not self._stop.is_set():
            try:
                item = self._submit.get(timeout=0.05 if eng.has_unfinished() else 0.5)
            except queue.Empty:
                item = None
            while item is not None:
                if self._stop.is_set():
                    return
                self._admit(item)
                try:
                    item = self._submit.get_nowait()
                except queue.Empty:
                    item = None
            if eng.has_unfinished():
                try:
                    if self.health is not None:
                        self.health.check()       # a dead peer rank: fail fast, no collective
                    eng.step()
                except Exception as e:  # fail every in-flight request, keep serving
                    self.errors += 1
                    for r in list(eng.running) + list(eng.waiting) + list(getattr(eng, "swapped", [])):
                        cb = getattr(r, "_on_done", None)
                        r._on_done = None          # reported here; _reap must not report it again
                        eng.abort(r.rid)
                        if cb:
                            cb(FinishReason.ERROR, str(e))
            self._reap()

    def _admit(self, item):
        if item[0] == "embed":
            _, ids, cb = item
            try:
                cb(self.engine.embed(ids), None)
            except Exception as e:
                cb(None, str(e))
            return
        _, cfg, push, done = item
        eng = self.engine
        tok = eng.tokenizer
        ids = cfg.prompt_ids if cfg.prompt_ids is not None else tok.encode(cfg.prompt)
        grammar = None
        if cfg.gbnf or cfg.json_mode:
            from ..structured.gbnf import GbnfConstraint
            if self._texts is None:
                self._texts = tok.token_texts()
            grammar = (GbnfConstraint.json_mode(self._texts) if cfg.json_mode
                       else GbnfConstraint.from_str(cfg.gbnf, self._texts))
            grammar.eos_id = eng.eos_id
        stop = StopChecker(cfg.stop, None, 1 << 30)
        params = SamplingParams(max_tokens=cfg.max_tokens, temperature=cfg.temperature, top_p=cfg.top_p,
                                top_k=cfg.top_k, repetition_penalty=cfg.repetition_penalty)

        def on_token(req, t):
            if t == eng.eos_id:
                return
            text = tok.decode_token(t)
            stop.push(t, text)
            push(TokenChunk(text, t))
            if stop.is_done():
                req.params.max_tokens = len(req.output_ids)
                req._stop_hit = True

        try:
            rid = eng.add_request(ids, params, on_token=on_token, grammar=grammar)
        except ValueError as e:
            done(FinishReason.ERROR, str(e))
            return
        for r in eng.waiting:
            if r.rid == rid:
                r._on_done = done

    def _reap(self):
        eng = self.engine
        for rid in list(eng.finished):
            r = eng.finished.pop(rid)
            cb = getattr(r, "_on_done", None)
            if cb is None:
                continue
            reason = r.finished
            if getattr(r, "_stop_hit", False) or reason == "stop":
                reason = FinishReason.STOP
            elif reason == "length":
                reason = FinishReason.LENGTH
            self.requests_served += 1
            cb(reason, None)

    # -- async side -----------------------------------------------------------------
    async def generate(self, config: GenerateConfig):
        loop = asyncio.get_running_loop()
        q: asyncio.Queue = asyncio.Queue()

        def post(item):
            try:
                loop.call_soon_threadsafe(q.put_nowait, item)
            except RuntimeError:           # the client's loop has closed (client went away)
                pass

        def push(chunk):
            post(chunk)

        def done(reason, err):
            post(TokenChunk(finish_reason=reason, error=err))

        self._submit.put(("gen", config, push, done))
        while True:
            chunk = await q.get()
            yield chunk
            if chunk.is_stop:
                return

    def embed(self, text: str) -> list[float]:
        """Mean-pooled final hidden state, computed on the engine thread."""
        ev = threading.Event()
        box = {}

        def cb(vec, err):
            box["v"], box["e"] = vec, err
            ev.set()

        self._submit.put(("embed", self.engine.tokenizer.encode(text), cb))
        ev.wait()
        if box["e"]:
            raise RuntimeError(box["e"])
        return box["v"]
