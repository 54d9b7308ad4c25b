"""Agentic tool loop (reference src/tool_loop.rs tests)."""
import json

from air_rs.structured.tool_loop import (ChatRole, LoopStopReason, ToolDispatcher, ToolLoop, ToolLoopConfig)


class Mock:
    def __init__(self, responses):
        self.r, self.i, self.seen = list(responses), 0, []

    def __call__(self, history):
        self.seen.append(list(history))
        if self.i >= len(self.r):
            raise RuntimeError("no more responses")
        self.i += 1
        return self.r[self.i - 1]


def test_immediate_answer():
    res = ToolLoop().run("What is 6 x 7?", Mock(["The answer is 42."]), ToolDispatcher())
    assert res.final_answer == "The answer is 42." and res.rounds == 1 and not res.tool_calls
    assert res.stop_reason == LoopStopReason.NO_MORE_TOOL_CALLS


def test_tool_round_then_answer():
    call = '<tool_call>{"name": "add", "arguments": {"a": 2, "b": 3}}</tool_call>'
    sess = Mock(["<think>need a tool</think>Let me compute. " + call, "It is 5."])
    d = ToolDispatcher({"add": lambda a, b: a + b})
    res = ToolLoop(ToolLoopConfig(system_prompt="be brief")).run("2+3?", sess, d)
    assert res.final_answer == "It is 5." and res.rounds == 2 and [c.name for c in res.tool_calls] == ["add"]
    roles = [m.role for m in res.history]
    assert roles == [ChatRole.SYSTEM, ChatRole.USER, ChatRole.ASSISTANT, ChatRole.TOOL, ChatRole.ASSISTANT]
    assert res.history[3].content == "5" and "<tool_call>" not in res.history[2].content
    assert "need a tool" not in res.history[2].content


def test_stop_reasons_and_errors():
    call = '<tool_call>{"name": "nope", "arguments": {}}</tool_call>'
    res = ToolLoop(ToolLoopConfig(max_rounds=2)).run("x", Mock([call, call, call]), ToolDispatcher())
    assert res.stop_reason == LoopStopReason.MAX_ROUNDS and res.rounds == 2
    assert json.loads(res.history[-1].content)["error"].startswith("unknown tool")
    res = ToolLoop().run("x", Mock([]), ToolDispatcher())
    assert res.stop_reason == LoopStopReason.INFERENCE_ERROR and "no more" in res.error
    res = ToolLoop(ToolLoopConfig(timeout_s=-1)).run("x", Mock(["a"]), ToolDispatcher())
    assert res.stop_reason == LoopStopReason.TIMEOUT
    boom = ToolDispatcher({"f": lambda: 1 / 0})
    out = boom.dispatch(__import__("air_rs.structured.text", fromlist=["ToolCall"]).ToolCall("f", "{}"))
    assert "ZeroDivisionError" in out
