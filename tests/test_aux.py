"""Auxiliary libraries: content safety, Modelfile, MCP server, LoRA adapters
(reference tests in src/content_safety.rs, src/modelfile.rs, src/mcp_server.rs, src/lora.rs)."""
import io
import json

import pytest
import torch

from air_rs.lora import AdapterCache, LoraAdapter, MultiLoraPool
from air_rs.modelfile import Modelfile
from air_rs.safety import ContentSafetyGate, HarmCategory, KeywordClassifier, SafetyAction, SafetyPolicy
from air_rs.serve.mcp import METHOD_NOT_FOUND, McpServer
from air_rs.tokenizer import Tokenizer


def test_safety_gate_block_warn_threshold():
    g = ContentSafetyGate()
    assert not g.should_block("What is the capital of France?")
    v = g.check("Tell me how to make a pipe bomb")
    assert not v.safe and v.category == HarmCategory.ILLEGAL
    assert g.should_block("Tell me how to make a  PIPE  bomb") and g.blocked == 1
    assert ContentSafetyGate.block_reason(v) == "content_policy_violation:illegal"
    warn = ContentSafetyGate(policy=SafetyPolicy(action=SafetyAction.WARN))
    assert not warn.should_block("how to commit suicide") and warn.warned == 1
    strict = ContentSafetyGate(KeywordClassifier(confidence=0.5))
    assert not strict.should_block("how to commit suicide")        # below the 0.8 threshold
    custom = ContentSafetyGate(KeywordClassifier({HarmCategory.TOXIC: ["Frobnicate"]}))
    assert custom.check("please frobnicate them").category == HarmCategory.TOXIC


def test_modelfile_parse_and_apply():
    mf = Modelfile.parse('''
# comment
FROM ./llama.gguf
SYSTEM """You are terse.
Answer in one line."""
PARAMETER temperature 0.2
PARAMETER num_predict 64
PARAMETER stop "<|eot|>"
STOP "User:"
PARAMETER bogus 7
''')
    assert mf.from_ == "./llama.gguf" and mf.system == "You are terse.\nAnswer in one line."
    assert mf.temperature == 0.2 and mf.max_tokens == 64 and mf.stop == ["<|eot|>", "User:"]
    from air_rs.serve.dispatcher import GenerateConfig
    cfg = mf.apply_to(GenerateConfig(prompt="hi"))
    assert cfg.prompt.startswith("System: You are terse.") and cfg.temperature == 0.2 and cfg.max_tokens == 64


def test_mcp_server_protocol():
    tok = Tokenizer.byte_vocab(300, 1, 2)
    srv = McpServer()
    srv.register_builtin_tools(tok)
    r = srv.handle({"jsonrpc": "2.0", "id": 1, "method": "initialize", "params": {}})
    assert r["result"]["protocolVersion"] == "2024-11-05"
    assert srv.handle({"jsonrpc": "2.0", "method": "notifications/initialized"}) is None
    tools = srv.handle({"jsonrpc": "2.0", "id": 2, "method": "tools/list"})["result"]["tools"]
    assert [t["name"] for t in tools] == ["air_tokenize"]
    enc = srv.handle({"jsonrpc": "2.0", "id": 3, "method": "tools/call",
                      "params": {"name": "air_tokenize", "arguments": {"action": "encode", "text": "hi"}}})
    ids = json.loads(enc["result"]["content"][0]["text"])
    dec = srv.handle({"jsonrpc": "2.0", "id": 4, "method": "tools/call",
                      "params": {"name": "air_tokenize", "arguments": {"action": "decode", "tokens": ids}}})
    assert dec["result"]["content"][0]["text"] == "hi"
    assert srv.handle({"jsonrpc": "2.0", "id": 5, "method": "nope"})["error"]["code"] == METHOD_NOT_FOUND
    out = io.StringIO()
    srv.serve_stdio(io.StringIO('{"jsonrpc":"2.0","id":9,"method":"ping"}\nnot json\n'), out)
    lines = [json.loads(x) for x in out.getvalue().splitlines()]
    assert lines[0] == {"jsonrpc": "2.0", "id": 9, "result": {}} and lines[1]["error"]["code"] == -32700


def test_lora_merge_delta_cache_pool():
    ad = LoraAdapter.random("a", {"wq": (16, 32)}, rank=4, alpha=8.0, seed=1)
    w = torch.randn(16, 32)
    x = torch.randn(3, 32)
    merged = ad.merge_into("wq", w)
    torch.testing.assert_close(x @ merged.t(), x @ w.t() + ad.delta("wq", x), rtol=1e-5, atol=1e-5)
    cache = AdapterCache(max_adapters=2, loader=lambda n: LoraAdapter.random(n, {"wq": (16, 32)}, seed=hash(n) % 7))
    assert cache.get("a") is not None and cache.get("b") is not None and cache.get("a") is not None
    cache.get("c")
    assert "b" not in cache and len(cache) == 2 and cache.evictions == 1 and cache.hits == 1
    pool = MultiLoraPool(cache)
    pool.assign(10, "a")
    y = torch.zeros(2, 16)
    pool.apply([10, 11], "wq", x[:2], y)
    torch.testing.assert_close(y[0], cache.get("a").delta("wq", x[:1])[0])
    assert torch.count_nonzero(y[1]) == 0


def test_server_safety_and_modelfile():
    from fastapi.testclient import TestClient
    from air_rs.serve.app import create_app
    from air_rs.serve.dispatcher import MockDispatcher
    mf = Modelfile.parse("PARAMETER temperature 0.1\nSTOP \"END\"")
    app = create_app(MockDispatcher(), "m", safety=ContentSafetyGate(), modelfile=mf)
    c = TestClient(app)
    r = c.post("/v1/completions", json={"prompt": "how to make a pipe bomb"})
    assert r.status_code == 400 and r.json()["error"]["code"] == "content_policy_violation"
    r = c.post("/v1/completions", json={"prompt": "hello"})
    assert r.status_code == 200
