"""Streaming text post-processing: stop strings, tool-call extraction, think tags.

Semantics follow the reference modules ``src/stop_seq.rs`` (rolling suffix buffer, longest
stop first, EOS before max-tokens before stop strings), ``src/tool_call.rs`` (Hermes
``<tool_call>{json}</tool_call>``, ``<|tool_call|>...<|end_tool_call|>``, Mistral
``[TOOL_CALLS] [...]`` and DeepSeek ``<｜tool▁call▁begin｜>name\\n{json}`` blocks; a block that
is not valid JSON yields ``name='?'`` with ``parse_error``) and ``src/think_tag.rs``
(``<think>...</think>`` split into reasoning and answer, streaming detectors by tag text or
by special token ids).
"""
from __future__ import annotations

import json
from collections import deque
from dataclasses import dataclass, field


# ---------------------------------------------------------------------------
# stop sequences
# ---------------------------------------------------------------------------

class StopReason:
    NOT_STOPPED = "not_stopped"
    MAX_TOKENS = "max_tokens"
    STOP_STRING = "stop_string"
    EOS = "eos"


class StopChecker:
    def __init__(self, stop_strings: list[str] | None = None, eos_token_id: int | None = None,
                 max_tokens: int = 1 << 30):
        self.stop_strings = sorted([s for s in (stop_strings or []) if s], key=len, reverse=True)
        self.eos_token_id = eos_token_id
        self.max_tokens = max_tokens
        self.capacity = 2 * max((len(s) for s in self.stop_strings), default=1) + 16
        self.reset()

    def reset(self):
        self.buffer: deque[str] = deque(maxlen=self.capacity)
        self.token_count = 0
        self.reason = StopReason.NOT_STOPPED
        self.matched: str | None = None
        self._parts: list[str] = []

    def push(self, token_id: int, text: str):
        if self.is_done():
            return
        self.token_count += 1
        self._parts.append(text)
        if self.eos_token_id is not None and token_id == self.eos_token_id:
            self.reason = StopReason.EOS
            return
        if self.token_count >= self.max_tokens:
            self.reason = StopReason.MAX_TOKENS
            return
        self.buffer.extend(text)
        tail = "".join(self.buffer)
        for s in self.stop_strings:
            if tail.endswith(s):
                self.reason = StopReason.STOP_STRING
                self.matched = s
                return

    def is_done(self) -> bool:
        return self.reason != StopReason.NOT_STOPPED

    @property
    def full_text(self) -> str:
        return "".join(self._parts)

    def strip_stop_suffix(self) -> str:
        t = self.full_text
        if self.reason == StopReason.STOP_STRING and self.matched and t.endswith(self.matched):
            return t[: -len(self.matched)]
        return t

    def holdback(self) -> int:
        """Characters a streaming client should withhold (a stop string may be forming)."""
        tail = "".join(self.buffer)
        best = 0
        for s in self.stop_strings:
            for k in range(min(len(s) - 1, len(tail)), 0, -1):
                if tail.endswith(s[:k]):
                    best = max(best, k)
                    break
        return best


# ---------------------------------------------------------------------------
# tool calls
# ---------------------------------------------------------------------------

@dataclass
class ToolCall:
    name: str
    arguments: str
    parse_error: bool = False

    def __str__(self):
        return f"{self.name}({self.arguments})"

    def to_openai(self, idx: int = 0) -> dict:
        return {"id": f"call_{idx}", "type": "function",
                "function": {"name": self.name, "arguments": self.arguments}}


@dataclass
class ParseResult:
    calls: list[ToolCall] = field(default_factory=list)
    remainder: str = ""

    def has_calls(self) -> bool:
        return bool(self.calls)


def _json_call(text: str) -> ToolCall:
    try:
        obj = json.loads(text.strip())
    except (json.JSONDecodeError, ValueError):
        return ToolCall("?", text.strip(), True)
    if not isinstance(obj, dict) or "name" not in obj:
        return ToolCall("?", text.strip(), True)
    args = obj.get("arguments", obj.get("parameters", {}))
    return ToolCall(str(obj["name"]), args if isinstance(args, str) else json.dumps(args))


def _extract(text: str, open_t: str, close_t: str, calls: list, parse) -> str:
    out = []
    i = 0
    while True:
        j = text.find(open_t, i)
        if j < 0:
            out.append(text[i:])
            break
        k = text.find(close_t, j + len(open_t))
        if k < 0:  # unterminated: take the rest as the block
            calls.append(parse(text[j + len(open_t):]))
            out.append(text[i:j])
            break
        calls.append(parse(text[j + len(open_t):k]))
        out.append(text[i:j])
        i = k + len(close_t)
    return "".join(out)


def _matching(text: str, open_c: str, close_c: str) -> int:
    depth, in_str, esc = 0, False, False
    for i, ch in enumerate(text):
        if in_str:
            if esc:
                esc = False
            elif ch == "\\":
                esc = True
            elif ch == '"':
                in_str = False
            continue
        if ch == '"':
            in_str = True
        elif ch == open_c:
            depth += 1
        elif ch == close_c:
            depth -= 1
            if depth == 0:
                return i
    return -1


def _deepseek(inner: str) -> ToolCall:
    t = inner.strip()
    nl = t.find("\n")
    if nl >= 0:
        first, rest = t[:nl].strip(), t[nl + 1:].strip()
        if first and not first.startswith("{"):
            return ToolCall(first, rest if rest.startswith("{") else "{}")
    return _json_call(t)


def parse_tool_calls(text: str) -> ParseResult:
    markers = ("<tool_call>", "<|tool_call|>", "[TOOL_CALLS]", "<｜tool▁call▁begin｜>")
    if not any(m in text for m in markers):
        return ParseResult([], text)
    calls: list[ToolCall] = []
    rem = _extract(text, "<tool_call>", "</tool_call>", calls, _json_call)
    rem = _extract(rem, "<|tool_call|>", "<|end_tool_call|>", calls, _json_call)
    p = rem.find("[TOOL_CALLS]")
    if p >= 0:
        after = rem[p + len("[TOOL_CALLS]"):]
        lead = len(after) - len(after.lstrip())
        body = after.lstrip()
        if body.startswith("["):
            end = _matching(body, "[", "]")
            if end >= 0:
                try:
                    arr = json.loads(body[:end + 1])
                    for obj in arr if isinstance(arr, list) else []:
                        calls.append(_json_call(json.dumps(obj)) if isinstance(obj, dict)
                                     else ToolCall("?", json.dumps(obj), True))
                except json.JSONDecodeError:
                    calls.append(ToolCall("?", body[:end + 1], True))
                rem = rem[:p] + after[lead + end + 1:]
    rem = _extract(rem, "<｜tool▁call▁begin｜>", "</tool_call>", calls, _deepseek)
    return ParseResult(calls, rem.strip())


def tool_call_parser(name: str):
    """CLI ``--tool-call-parser`` values map onto the one multi-format parser."""
    if name not in ("hermes", "mistral", "llama3_json", "llama", "deepseek", "auto", "pythonic"):
        raise ValueError(f"unknown tool-call parser {name!r}")
    return parse_tool_calls


# ---------------------------------------------------------------------------
# think tags
# ---------------------------------------------------------------------------

THINK_OPEN, THINK_CLOSE = "<think>", "</think>"


@dataclass
class ThinkResult:
    thinking: str
    output: str

    def is_pure_output(self) -> bool:
        return not self.thinking


def strip_think_tags(text: str) -> ThinkResult:
    thinking, out, i = [], [], 0
    while True:
        j = text.find(THINK_OPEN, i)
        if j < 0:
            out.append(text[i:])
            break
        out.append(text[i:j])
        k = text.find(THINK_CLOSE, j + len(THINK_OPEN))
        if k < 0:  # still thinking
            thinking.append(text[j + len(THINK_OPEN):])
            break
        thinking.append(text[j + len(THINK_OPEN):k])
        i = k + len(THINK_CLOSE)
    return ThinkResult("".join(thinking).strip(), "".join(out).strip())


class ThinkState:
    """Incremental split of a token stream into reasoning and answer."""

    def __init__(self):
        self.buf = ""

    def push_token(self, token: str):
        self.buf += token

    def finish(self) -> ThinkResult:
        return strip_think_tags(self.buf)


class ThinkEvent:
    ENTER = "enter"
    EXIT = "exit"


class TagBasedThinking:
    def __init__(self):
        self.reset()

    def reset(self):
        self._in = False
        self._tail = ""

    def process_token(self, token_id: int, text: str):
        self._tail = (self._tail + text)[-16:]
        if not self._in and self._tail.endswith(THINK_OPEN):
            self._in = True
            return ThinkEvent.ENTER
        if self._in and self._tail.endswith(THINK_CLOSE):
            self._in = False
            return ThinkEvent.EXIT
        return None

    def in_think_block(self) -> bool:
        return self._in


class SpecialTokenThinking:
    def __init__(self, start_ids=(), end_ids=()):
        self.start_ids, self.end_ids = set(start_ids), set(end_ids)
        self._in = False

    @classmethod
    def from_vocab(cls, tokens: list[str]) -> "SpecialTokenThinking":
        starts = {i for i, t in enumerate(tokens) if t in ("<think>", "<|think|>", "<start_of_thought>")}
        ends = {i for i, t in enumerate(tokens) if t in ("</think>", "<|/think|>", "<end_of_thought>")}
        return cls(starts, ends)

    def reset(self):
        self._in = False

    def process_token(self, token_id: int, text: str = ""):
        if token_id in self.start_ids and not self._in:
            self._in = True
            return ThinkEvent.ENTER
        if token_id in self.end_ids and self._in:
            self._in = False
            return ThinkEvent.EXIT
        return None

    def in_think_block(self) -> bool:
        return self._in
