"""Public Python API, same names and signatures as the reference's ``air_rs`` package
(``python/air_rs/_air_rs.pyi``, ``src/python.rs:81-650``): ``Engine.from_gguf``, ``generate``,
``stream_to_list``, ``_stream_channel``, ``set_grammar`` / ``clear_grammar`` / ``has_grammar``,
``reset``, ``metrics``; ``GenerateConfig``; ``GbnfConstraint`` builders; ``Metrics``;
``TokenChannel``.

Differences that are fixes: per-call ``temperature`` / ``top_p`` / ``top_k`` /
``repetition_penalty`` / ``stop_strings`` are honoured (the reference reads them but only
applies ``max_tokens`` and the grammar, ``src/python.rs:413-421``), and ``_stream_channel``
delivers tokens while they are generated instead of after the whole generation.
"""
from __future__ import annotations

import os
import queue
import threading
import time
from dataclasses import dataclass, field

from .runtime.engine import Engine as _CoreEngine, SamplingParams
from .structured.gbnf import GbnfConstraint as _Constraint, GbnfGrammar, GbnfError
from .structured.text import StopChecker


class GenerateConfig:
    """Sampling parameters for a single generation call."""

    def __init__(self, *, max_tokens: int = 512, temperature: float = 0.7, top_p: float = 0.9,
                 top_k: int = 40, repetition_penalty: float = 1.1, stop_strings: list[str] | None = None,
                 grammar: "GbnfConstraint | None" = None):
        self.max_tokens = int(max_tokens)
        self.temperature = float(temperature)
        self.top_p = float(top_p)
        self.top_k = int(top_k)
        self.repetition_penalty = float(repetition_penalty)
        self.stop_strings = list(stop_strings or [])
        self.grammar = grammar

    def __repr__(self):
        return (f"GenerateConfig(max_tokens={self.max_tokens}, temperature={self.temperature}, "
                f"top_p={self.top_p}, top_k={self.top_k}, repetition_penalty={self.repetition_penalty}, "
                f"stop_strings={self.stop_strings!r}, grammar={self.grammar!r})")

    def sampling(self, ignore_eos: bool = False) -> SamplingParams:
        return SamplingParams(max_tokens=self.max_tokens, temperature=self.temperature, top_p=self.top_p,
                              top_k=self.top_k, repetition_penalty=self.repetition_penalty,
                              ignore_eos=ignore_eos)


class GbnfConstraint:
    """A grammar specification; bound to an engine's vocabulary at generation time."""

    def __init__(self, kind: str, payload=None):
        self._kind = kind
        self._payload = payload

    @classmethod
    def json_mode(cls) -> "GbnfConstraint":
        return cls("json")

    @classmethod
    def integer(cls) -> "GbnfConstraint":
        return cls("integer")

    @classmethod
    def identifier(cls) -> "GbnfConstraint":
        return cls("identifier")

    @classmethod
    def choice(cls, options: list[str]) -> "GbnfConstraint":
        if not options:
            raise ValueError("choice() requires at least one option")
        return cls("choice", list(options))

    @classmethod
    def from_grammar(cls, grammar: str) -> "GbnfConstraint":
        try:
            GbnfGrammar.parse(grammar)
        except GbnfError as e:
            raise ValueError(f"Invalid GBNF grammar: {e}") from e
        return cls("raw", grammar)

    def build(self, token_texts: list[str]) -> _Constraint:
        if self._kind == "json":
            return _Constraint.json_mode(token_texts)
        if self._kind == "integer":
            return _Constraint.integer(token_texts)
        if self._kind == "identifier":
            return _Constraint.identifier(token_texts)
        if self._kind == "choice":
            return _Constraint.choice(self._payload, token_texts)
        return _Constraint.from_str(self._payload, token_texts)

    def __repr__(self):
        if self._kind == "raw":
            return f"GbnfConstraint.from_grammar({self._payload!r})"
        if self._kind == "choice":
            return f"GbnfConstraint.choice({self._payload!r})"
        return f"GbnfConstraint.{ {'json': 'json_mode'}.get(self._kind, self._kind)}()"


@dataclass(frozen=True)
class Metrics:
    """Read-only metrics snapshot of the last generation."""
    tokens_per_second: float = 0.0
    time_to_first_token_ms: float = 0.0
    total_time_ms: float = 0.0
    prompt_tokens: int = 0
    generated_tokens: int = 0

    def __repr__(self):
        return (f"Metrics(tokens_per_second={self.tokens_per_second:.2f}, "
                f"time_to_first_token_ms={self.time_to_first_token_ms:.2f}, "
                f"total_time_ms={self.total_time_ms:.2f}, prompt_tokens={self.prompt_tokens}, "
                f"generated_tokens={self.generated_tokens})")


class TokenChannel:
    """Per-request token stream (returned by ``Engine._stream_channel``)."""

    _DONE = object()

    def __init__(self):
        self._q: queue.Queue = queue.Queue()
        self._error: BaseException | None = None

    def _put(self, tok: str):
        self._q.put(tok)

    def _close(self, error: BaseException | None = None):
        self._error = error
        self._q.put(self._DONE)

    def recv_sync(self) -> str | None:
        item = self._q.get()
        if item is self._DONE:
            self._q.put(self._DONE)  # stay closed for later calls
            if self._error is not None:
                raise RuntimeError(f"generation failed: {self._error}") from self._error
            return None
        return item

    def recv_or_stop(self) -> str:
        tok = self.recv_sync()
        if tok is None:
            raise StopAsyncIteration
        return tok

    def __iter__(self):
        while True:
            t = self.recv_sync()
            if t is None:
                return
            yield t


class Engine:
    """High-performance LLM inference engine (B200 / CUDA, or the CPU oracle)."""

    def __init__(self, core: _CoreEngine, defaults: GenerateConfig, path: str = ""):
        self._core = core
        self._defaults = defaults
        self._grammar: GbnfConstraint | None = None
        self._lock = threading.Lock()
        self._metrics = Metrics()
        self._token_texts: list[str] | None = None
        self.path = path

    # -- construction -----------------------------------------------------
    @classmethod
    def from_gguf(cls, path: str, *, temperature: float = 0.7, top_p: float = 0.9, top_k: int = 40,
                  repetition_penalty: float = 1.1, resident: bool = True, council: bool = False,
                  epsilon: float = 0.15, device: str | None = None, max_batch: int = 64,
                  max_model_len: int | None = None, **kw) -> "Engine":
        from .runtime.builder import engine_from_gguf
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        core = engine_from_gguf(path, device=device, max_batch=max_batch, max_model_len=max_model_len, **kw)
        d = GenerateConfig(temperature=temperature, top_p=top_p, top_k=top_k,
                           repetition_penalty=repetition_penalty)
        eng = cls(core, d, path)
        eng.council, eng.epsilon, eng.resident = council, epsilon, resident
        return eng

    @classmethod
    def from_core(cls, core: _CoreEngine, **defaults) -> "Engine":
        return cls(core, GenerateConfig(**defaults))

    # -- grammar ------------------------------------------------------------
    def set_grammar(self, constraint: GbnfConstraint) -> None:
        self._grammar = constraint

    def clear_grammar(self) -> None:
        self._grammar = None

    def has_grammar(self) -> bool:
        return self._grammar is not None

    def _texts(self) -> list[str]:
        if self._token_texts is None:
            self._token_texts = self._core.tokenizer.token_texts()
        return self._token_texts

    # -- generation -----------------------------------------------------------
    def _config(self, config: GenerateConfig | None) -> GenerateConfig:
        if config is None:
            d = self._defaults
            return GenerateConfig(max_tokens=d.max_tokens, temperature=d.temperature, top_p=d.top_p,
                                  top_k=d.top_k, repetition_penalty=d.repetition_penalty)
        return config

    def _run(self, prompt: str, config: GenerateConfig | None, on_text=None) -> str:
        cfg = self._config(config)
        tok = self._core.tokenizer
        ids = tok.encode(prompt)
        spec = cfg.grammar or self._grammar
        grammar = spec.build(self._texts()) if spec is not None else None
        if grammar is not None:
            grammar.eos_id = self._core.eos_id
        stop = StopChecker(cfg.stop_strings, None, cfg.max_tokens + 1)
        parts: list[str] = []
        t0 = time.perf_counter()
        first = [None]

        def on_token(req, t):
            if first[0] is None:
                first[0] = time.perf_counter()
            if t == self._core.eos_id:
                return
            text = tok.decode_token(t)
            stop.push(t, text)
            parts.append(text)
            if on_text is not None:
                on_text(text)
            if stop.is_done():
                req.params.max_tokens = len(req.output_ids)  # finish after this token

        with self._lock:
            rid = self._core.add_request(ids, cfg.sampling(), on_token=on_token, grammar=grammar)
            while self._core.has_unfinished():
                self._core.step()
            req = self._core.finished.pop(rid)
        t1 = time.perf_counter()
        n = len(req.output_ids)
        ttft = ((first[0] or t1) - t0) * 1e3
        tps = (n - 1) / (t1 - first[0]) if first[0] and n > 1 and t1 > first[0] else 0.0
        self._metrics = Metrics(tps, ttft, (t1 - t0) * 1e3, len(req.prompt_ids), n)
        text = "".join(parts)
        if stop.reason == "stop_string" and stop.matched and text.endswith(stop.matched):
            text = text[: -len(stop.matched)]
        return text

    def generate(self, prompt: str, config: GenerateConfig | None = None) -> str:
        return self._run(prompt, config)

    def stream_to_list(self, prompt: str, config: GenerateConfig | None = None) -> list[str]:
        out: list[str] = []
        self._run(prompt, config, on_text=out.append)
        return out

    def _stream_channel(self, prompt: str, config: GenerateConfig | None = None) -> TokenChannel:
        ch = TokenChannel()

        def work():
            try:
                self._run(prompt, config, on_text=ch._put)
                ch._close()
            except BaseException as e:  # surfaced to the consumer by recv_sync
                ch._close(e)

        threading.Thread(target=work, name="air_rs_generate", daemon=True).start()
        return ch

    def reset(self) -> None:
        """Drop all cached sequence state (KV blocks of any unfinished request)."""
        with self._lock:
            for r in list(self._core.running) + list(self._core.waiting):
                self._core.abort(r.rid)
            self._core.finished.clear()
            if self._core.oracle is not None:
                self._core.oracle.reset()

    def metrics(self) -> Metrics:
        return self._metrics

    @property
    def core(self) -> _CoreEngine:
        return self._core
