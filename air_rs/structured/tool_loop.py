"""Agentic tool loop (reference ``src/tool_loop.rs``: ChatMessage / ChatRole, ToolDispatcher,
ToolLoopConfig {max_rounds 10, timeout 300 s, system prompt, strip thinking, strip tool-call
blocks from the visible text}, ToolLoop.run -> ToolLoopResult with the stop reason).

Each round renders the history, generates, strips ``<think>`` blocks, parses tool calls
(hermes / mistral / llama / deepseek formats), runs them through the dispatcher and appends
their results as tool messages; a reply without tool calls is the final answer.
``EngineSession`` generates through ``air_rs.api.Engine`` with a chat template.
"""
from __future__ import annotations

import enum
import json
import time
from dataclasses import dataclass, field
from typing import Callable

from .text import ToolCall, parse_tool_calls, strip_think_tags


class ChatRole(str, enum.Enum):
    SYSTEM = "system"
    USER = "user"
    ASSISTANT = "assistant"
    TOOL = "tool"


@dataclass
class ChatMessage:
    role: ChatRole
    content: str
    tool_call_id: str | None = None

    @classmethod
    def system(cls, c: str):
        return cls(ChatRole.SYSTEM, c)

    @classmethod
    def user(cls, c: str):
        return cls(ChatRole.USER, c)

    @classmethod
    def assistant(cls, c: str):
        return cls(ChatRole.ASSISTANT, c)

    @classmethod
    def tool_result(cls, call_id: str, c: str):
        return cls(ChatRole.TOOL, c, call_id)

    def as_dict(self) -> dict:
        d = {"role": self.role.value, "content": self.content}
        if self.tool_call_id:
            d["tool_call_id"] = self.tool_call_id
        return d


class ToolDispatcher:
    """Maps tool names to callables taking the parsed JSON arguments; a callable may also be
    given for every call (``FnDispatcher`` in the reference)."""

    def __init__(self, tools: dict[str, Callable] | None = None, fallback: Callable | None = None):
        self.tools = dict(tools or {})
        self.fallback = fallback

    def dispatch(self, call: ToolCall) -> str:
        if call.parse_error:
            return json.dumps({"error": f"could not parse arguments of {call.name}"})
        fn = self.tools.get(call.name)
        try:
            args = json.loads(call.arguments) if call.arguments else {}
        except json.JSONDecodeError:
            args = call.arguments
        if fn is None:
            if self.fallback is None:
                return json.dumps({"error": f"unknown tool {call.name}"})
            return str(self.fallback(call))
        try:
            out = fn(**args) if isinstance(args, dict) else fn(args)
        except Exception as e:   # tool errors go back to the model as the tool's result
            return json.dumps({"error": f"{type(e).__name__}: {e}"})
        return out if isinstance(out, str) else json.dumps(out)


class LoopStopReason(str, enum.Enum):
    NO_MORE_TOOL_CALLS = "no_more_tool_calls"
    MAX_ROUNDS = "max_rounds"
    TIMEOUT = "timeout"
    INFERENCE_ERROR = "inference_error"


@dataclass
class ToolLoopConfig:
    max_rounds: int = 10
    timeout_s: float = 300.0
    system_prompt: str | None = None
    strip_thinking: bool = True
    strip_tool_calls_from_visible: bool = True


@dataclass
class ToolLoopResult:
    final_answer: str
    rounds: int
    tool_calls: list[ToolCall]
    history: list[ChatMessage]
    stop_reason: LoopStopReason
    error: str | None = None


class ToolLoop:
    def __init__(self, config: ToolLoopConfig | None = None):
        self.config = config or ToolLoopConfig()

    @staticmethod
    def _last_assistant(history: list[ChatMessage]) -> str:
        for m in reversed(history):
            if m.role == ChatRole.ASSISTANT:
                return m.content
        return ""

    def run(self, user_message: str, session: Callable[[list[ChatMessage]], str],
            dispatcher: ToolDispatcher) -> ToolLoopResult:
        cfg = self.config
        t0 = time.monotonic()
        history: list[ChatMessage] = []
        if cfg.system_prompt:
            history.append(ChatMessage.system(cfg.system_prompt))
        history.append(ChatMessage.user(user_message))
        calls_all: list[ToolCall] = []
        rounds = 0

        def done(reason, err=None, answer=None):
            return ToolLoopResult(answer if answer is not None else self._last_assistant(history), rounds,
                                  calls_all, history, reason, err)
        while True:
            if time.monotonic() - t0 > cfg.timeout_s:
                return done(LoopStopReason.TIMEOUT)
            if rounds >= cfg.max_rounds:
                return done(LoopStopReason.MAX_ROUNDS)
            try:
                raw = session(history)
            except Exception as e:
                return done(LoopStopReason.INFERENCE_ERROR, str(e))
            rounds += 1
            text = strip_think_tags(raw).output if cfg.strip_thinking else raw
            parsed = parse_tool_calls(text)
            if not parsed.calls:
                history.append(ChatMessage.assistant(parsed.remainder))
                return done(LoopStopReason.NO_MORE_TOOL_CALLS, answer=parsed.remainder)
            history.append(ChatMessage.assistant(parsed.remainder if cfg.strip_tool_calls_from_visible else text))
            for i, call in enumerate(parsed.calls):
                calls_all.append(call)
                history.append(ChatMessage.tool_result(f"call_{rounds}_{i}", dispatcher.dispatch(call)))


class EngineSession:
    """A session generating with ``air_rs.api.Engine`` over a chat-template rendering."""

    def __init__(self, engine, template: str = "chatml", **gen_kw):
        self.engine, self.template, self.gen_kw = engine, template, gen_kw

    def __call__(self, history: list[ChatMessage]) -> str:
        from ..utils import format_chat
        msgs = [m.as_dict() for m in history]
        for m in msgs:
            if m["role"] == "tool":
                m["role"] = "user"
                m["content"] = f"<tool_response>\n{m['content']}\n</tool_response>"
        return self.engine.generate(format_chat(msgs, self.template), **self.gen_kw)
