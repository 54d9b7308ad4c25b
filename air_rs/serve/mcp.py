"""Model Context Protocol server (reference ``src/mcp_server.rs``): JSON-RPC 2.0 over stdio
with ``initialize`` / ``ping`` / ``tools/list`` / ``tools/call``, and built-in tools
``air_tokenize`` (encode / decode), ``air_model_info`` and ``air_generate`` (which runs the
loaded engine; the reference registers only the tokenizer tool).
"""
from __future__ import annotations

import json
import sys
from dataclasses import dataclass
from typing import Callable

PARSE_ERROR, INVALID_REQUEST, METHOD_NOT_FOUND, INVALID_PARAMS, INTERNAL_ERROR = -32700, -32600, -32601, -32602, -32603
PROTOCOL_VERSION = "2024-11-05"


def ok(id_, result) -> dict:
    return {"jsonrpc": "2.0", "id": id_, "result": result}


def err(id_, code: int, message: str) -> dict:
    return {"jsonrpc": "2.0", "id": id_, "error": {"code": code, "message": message}}


def text_content(t: str) -> dict:
    return {"type": "text", "text": t}


@dataclass
class McpTool:
    name: str
    description: str
    input_schema: dict
    handler: Callable[[dict], dict]

    def descriptor(self) -> dict:
        return {"name": self.name, "description": self.description, "inputSchema": self.input_schema}


class McpServer:
    def __init__(self, name: str = "air-rs", version: str | None = None):
        from .. import __version__
        self.name, self.version = name, version or __version__
        self.tools: dict[str, McpTool] = {}

    def register_tool(self, tool: McpTool):
        self.tools[tool.name] = tool

    def register_builtin_tools(self, tokenizer=None, engine=None, model_name: str = "air-rs"):
        if tokenizer is not None:
            def tokenize(args):
                act = args.get("action")
                if act == "encode":
                    return {"content": [text_content(json.dumps(tokenizer.encode(args.get("text", ""))))]}
                if act == "decode":
                    return {"content": [text_content(tokenizer.decode([int(t) for t in args.get("tokens", [])]))]}
                return {"content": [text_content("action must be 'encode' or 'decode'")], "isError": True}
            self.register_tool(McpTool(
                "air_tokenize", "Encode text to token ids or decode token ids to text with the model's tokenizer.",
                {"type": "object", "properties": {"action": {"type": "string", "enum": ["encode", "decode"]},
                                                  "text": {"type": "string"},
                                                  "tokens": {"type": "array", "items": {"type": "integer"}}},
                 "required": ["action"]}, tokenize))
        if engine is not None:
            cfg = engine.cfg

            def info(args):
                d = {"model": model_name, "layers": cfg.n_layers, "hidden": cfg.hidden_dim, "heads": cfg.n_heads,
                     "kv_heads": cfg.n_kv_heads, "vocab": cfg.vocab_size, "experts": cfg.n_experts,
                     "device": "cuda" if engine.runner is not None else "cpu"}
                return {"content": [text_content(json.dumps(d))]}
            self.register_tool(McpTool("air_model_info", "Architecture of the loaded model.",
                                       {"type": "object", "properties": {}}, info))

            def generate(args):
                from ..runtime.engine import SamplingParams
                tok = tokenizer or engine.tokenizer
                ids = tok.encode(str(args.get("prompt", "")))
                sp = SamplingParams(max_tokens=int(args.get("max_tokens", 64)),
                                    temperature=float(args.get("temperature", 0.0)))
                out = engine.generate_ids([ids], sp)[0]
                return {"content": [text_content(tok.decode(out))]}
            self.register_tool(McpTool(
                "air_generate", "Generate a completion with the loaded model.",
                {"type": "object", "properties": {"prompt": {"type": "string"}, "max_tokens": {"type": "integer"},
                                                  "temperature": {"type": "number"}}, "required": ["prompt"]},
                generate))

    def handle(self, req) -> dict | None:
        """One JSON-RPC request (dict) -> response dict (None for notifications)."""
        if not isinstance(req, dict) or req.get("jsonrpc") != "2.0" or "method" not in req:
            return err(req.get("id") if isinstance(req, dict) else None, INVALID_REQUEST, "invalid request")
        id_, m, params = req.get("id"), req["method"], req.get("params") or {}
        if m == "initialize":
            return ok(id_, {"protocolVersion": PROTOCOL_VERSION,
                            "capabilities": {"tools": {"listChanged": False}},
                            "serverInfo": {"name": self.name, "version": self.version}})
        if m in ("initialized", "notifications/initialized"):
            return None if id_ is None else ok(id_, None)
        if m == "ping":
            return ok(id_, {})
        if m == "tools/list":
            return ok(id_, {"tools": [t.descriptor() for t in self.tools.values()]})
        if m == "tools/call":
            name = params.get("name")
            if not name:
                return err(id_, INVALID_PARAMS, "missing 'name' in tools/call params")
            tool = self.tools.get(name)
            if tool is None:
                return err(id_, METHOD_NOT_FOUND, f"tool not found: {name}")
            try:
                return ok(id_, tool.handler(params.get("arguments") or {}))
            except Exception as e:  # tool failures are results, not protocol errors
                return ok(id_, {"content": [text_content(f"{type(e).__name__}: {e}")], "isError": True})
        return err(id_, METHOD_NOT_FOUND, f"method not found: {m}")

    def handle_line(self, line: str) -> str | None:
        try:
            req = json.loads(line)
        except json.JSONDecodeError as e:
            return json.dumps(err(None, PARSE_ERROR, f"parse error: {e}"))
        resp = self.handle(req)
        return None if resp is None else json.dumps(resp)

    def serve_stdio(self, stdin=None, stdout=None):
        stdin, stdout = stdin or sys.stdin, stdout or sys.stdout
        for line in stdin:
            if not line.strip():
                continue
            out = self.handle_line(line)
            if out is not None:
                stdout.write(out + "\n")
                stdout.flush()
