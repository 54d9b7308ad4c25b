"""OpenAI-compatible REST server (reference ``src/api.rs:861-882`` routes).

Routes: ``/v1/chat/completions``, ``/v1/completions``, ``/v1/embeddings``, ``/v1/responses``,
``/v1/models``, ``/v1/models/{id}`` and their un-versioned aliases, ``/health`` and
``/metrics`` (Prometheus text). Chat requests are rendered with the model family's chat
template over the whole conversation (the reference passes only the last message's content,
``src/api.rs:461``). Streaming responses are Server-Sent Events, one chunk per token,
terminated by ``data: [DONE]``.
"""
from __future__ import annotations

import json
import time

from fastapi import FastAPI, Request
from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse

from .. import __version__
from ..structured.chat_template import ChatTemplate, detect_format
from ..structured.text import parse_tool_calls, strip_think_tags
from .dispatcher import Dispatcher, GenerateConfig
from .openai import (ApiError, ApiErrorCode, ApiKeyStore, PrometheusMetrics, RateLimiter, chat_chunk, new_id,
                     now, stop_list, to_sse, usage, validate_sampling)

DEFAULT_MAX_TOKENS = 128       # reference: req.max_tokens.unwrap_or(128)
DEFAULT_TEMPERATURE = 0.7      # reference default_temperature()


def create_app(dispatcher: Dispatcher, model_name: str = "air-rs", *, api_keys: list[str] | None = None,
               rate_limit: tuple[float, int] | None = None, chat_format: str | None = None,
               reasoning_format: str | None = None, tool_call_parser: str | None = None,
               safety=None, modelfile=None) -> FastAPI:
    """``safety``: an ``air_rs.safety.ContentSafetyGate`` screening prompts (and completed
    outputs); ``modelfile``: an ``air_rs.modelfile.Modelfile`` supplying defaults."""
    app = FastAPI(title="air-rs", version=__version__)
    keys = ApiKeyStore(api_keys)
    limiter = RateLimiter(*rate_limit) if rate_limit else None
    metrics = PrometheusMetrics()
    template = ChatTemplate(chat_format or detect_format(model_name))
    state = {"start": time.time(), "served": 0}

    @app.exception_handler(ApiError)
    async def _api_error(request: Request, exc: ApiError):
        return JSONResponse(exc.body(), status_code=exc.status)

    async def guard(request: Request) -> dict:
        if not keys.check(request.headers.get("authorization")):
            raise ApiError("Invalid API key", ApiErrorCode.AUTHENTICATION, "invalid_api_key")
        client = request.headers.get("authorization") or (request.client.host if request.client else "anon")
        if limiter is not None and not limiter.allow(client):
            raise ApiError("Rate limit exceeded", ApiErrorCode.RATE_LIMIT, "rate_limit_exceeded")
        try:
            body = await request.json()
        except (json.JSONDecodeError, ValueError):
            raise ApiError("Request body is not valid JSON")
        if not isinstance(body, dict):
            raise ApiError("Request body must be a JSON object")
        model = body.get("model") or model_name
        if model not in dispatcher.list_models() and model != model_name:
            raise ApiError.model_not_found(model)
        validate_sampling(body)
        return body

    def screen(text: str):
        if safety is not None and safety.policy.screen_input and safety.should_block(text):
            raise ApiError(safety.block_reason(safety.check(text)), ApiErrorCode.INVALID_REQUEST,
                           "content_policy_violation")

    def screen_output(text: str) -> str:
        if safety is not None and safety.policy.screen_output and safety.should_block(text):
            raise ApiError(safety.block_reason(safety.check(text)), ApiErrorCode.INVALID_REQUEST,
                           "content_policy_violation")
        return text

    def config_from(body: dict, prompt: str, max_key: str = "max_tokens") -> GenerateConfig:
        screen(prompt)
        if modelfile is not None:
            mf_cfg = modelfile.apply_to(GenerateConfig(model=model_name, prompt=prompt))
            prompt = mf_cfg.prompt
            for k in ("temperature", "top_p", "max_tokens"):
                if body.get(k) is None and getattr(modelfile, k) is not None:
                    body = {**body, k: getattr(mf_cfg, k)}
            if modelfile.stop and not body.get("stop"):
                body = {**body, "stop": list(modelfile.stop)}
        rf = body.get("response_format") or {}
        return GenerateConfig(
            model=body.get("model") or model_name, prompt=prompt,
            max_tokens=int(body.get(max_key) or DEFAULT_MAX_TOKENS),
            temperature=float(body["temperature"]) if body.get("temperature") is not None else DEFAULT_TEMPERATURE,
            top_p=float(body.get("top_p") or 1.0), top_k=int(body.get("top_k") or 0),
            repetition_penalty=float(body.get("repetition_penalty") or 1.0),
            stop=stop_list(body.get("stop")), gbnf=body.get("gbnf") or body.get("grammar"),
            json_mode=rf.get("type") == "json_object")

    async def run(cfg: GenerateConfig):
        """Collects a whole completion: (text, n_tokens, finish_reason, ttft_ms)."""
        t0 = time.perf_counter()
        parts, ttft, reason = [], None, "stop"
        metrics.active_requests += 1
        try:
            async for ch in dispatcher.generate(cfg):
                if ch.is_stop:
                    if ch.error:
                        metrics.requests_failed += 1
                        raise ApiError(ch.error, ApiErrorCode.SERVER_ERROR)
                    reason = ch.finish_reason
                    break
                if ttft is None:
                    ttft = (time.perf_counter() - t0) * 1e3
                parts.append(ch.text)
        finally:
            metrics.active_requests -= 1
        metrics.latency.record((time.perf_counter() - t0) * 1e3)
        if ttft is not None:
            metrics.ttft.record(ttft)
        metrics.requests_total += 1
        metrics.tokens_generated += len(parts)
        state["served"] += 1
        return "".join(parts), len(parts), reason

    def stream(cfg: GenerateConfig, make_chunk, final_chunk):
        async def gen():
            t0 = time.perf_counter()
            first = True
            n = 0
            metrics.active_requests += 1
            try:
                async for ch in dispatcher.generate(cfg):
                    if ch.is_stop:
                        if ch.error:
                            metrics.requests_failed += 1
                            yield to_sse(ApiError(ch.error, ApiErrorCode.SERVER_ERROR).body())
                        else:
                            yield to_sse(final_chunk(ch.finish_reason))
                        break
                    if first:
                        metrics.ttft.record((time.perf_counter() - t0) * 1e3)
                        first = False
                    n += 1
                    yield to_sse(make_chunk(ch.text))
                yield "data: [DONE]\n\n"
            finally:
                metrics.active_requests -= 1
                metrics.requests_total += 1
                metrics.tokens_generated += n
                metrics.latency.record((time.perf_counter() - t0) * 1e3)
                state["served"] += 1
        return StreamingResponse(gen(), media_type="text/event-stream")

    # ------------------------------------------------------------------ routes
    async def chat_completions(request: Request):
        body = await guard(request)
        msgs = body.get("messages")
        if not isinstance(msgs, list) or not msgs:
            raise ApiError("messages must be a non-empty list")
        for m in msgs:
            if not isinstance(m, dict) or "role" not in m:
                raise ApiError("each message needs a role")
            if isinstance(m.get("content"), list):  # content parts -> text
                m["content"] = "".join(p.get("text", "") for p in m["content"] if isinstance(p, dict))
        prompt = template.apply(msgs)
        cfg = config_from(body, prompt)
        model = cfg.model
        cid = new_id("chatcmpl")
        metrics.prompt_tokens += dispatcher.count_tokens(prompt)
        if body.get("stream"):
            first = {"sent": False}

            def mk(text):
                delta = {"content": text}
                if not first["sent"]:
                    delta["role"] = "assistant"
                    first["sent"] = True
                return chat_chunk(cid, model, delta)
            return stream(cfg, mk, lambda r: chat_chunk(cid, model, {}, r))
        text, n, reason = await run(cfg)
        text = screen_output(text)
        msg = {"role": "assistant", "content": text}
        if reasoning_format and reasoning_format != "none":
            tr = strip_think_tags(text)
            msg["content"], msg["reasoning_content"] = tr.output, tr.thinking or None
        if tool_call_parser or body.get("tools"):
            pr = parse_tool_calls(msg["content"])
            if pr.has_calls():
                msg["content"] = pr.remainder or None
                msg["tool_calls"] = [c.to_openai(i) for i, c in enumerate(pr.calls)]
                reason = "tool_calls"
        return {"id": cid, "object": "chat.completion", "created": now(), "model": model,
                "choices": [{"index": 0, "message": msg, "finish_reason": reason}],
                "usage": usage(dispatcher.count_tokens(prompt), n)}

    async def completions(request: Request):
        body = await guard(request)
        prompt = body.get("prompt")
        if isinstance(prompt, list):
            prompt = "".join(prompt)
        if not isinstance(prompt, str):
            raise ApiError("prompt must be a string")
        cfg = config_from(body, prompt)
        cid = new_id("cmpl")
        metrics.prompt_tokens += dispatcher.count_tokens(prompt)

        def chunk(text, reason=None):
            return {"id": cid, "object": "text_completion", "created": now(), "model": cfg.model,
                    "choices": [{"index": 0, "text": text, "finish_reason": reason}]}
        if body.get("stream"):
            return stream(cfg, chunk, lambda r: chunk("", r))
        text, n, reason = await run(cfg)
        out = chunk(screen_output(text), reason)
        out["usage"] = usage(dispatcher.count_tokens(prompt), n)
        return out

    async def embeddings(request: Request):
        body = await guard(request)
        inp = body.get("input")
        items = [inp] if isinstance(inp, str) else inp
        if not isinstance(items, list) or not items or not all(isinstance(s, str) for s in items):
            raise ApiError("input must be a string or a list of strings")
        import asyncio
        data = []
        for i, s in enumerate(items):
            vec = await asyncio.get_running_loop().run_in_executor(None, dispatcher.embed, s)
            data.append({"object": "embedding", "embedding": vec, "index": i})
        n = sum(dispatcher.count_tokens(s) for s in items)
        return {"object": "list", "data": data, "model": body.get("model") or model_name, "usage": usage(n, 0)}

    async def responses(request: Request):
        body = await guard(request)
        inp = body.get("input")
        if isinstance(inp, str):
            msgs = [{"role": "user", "content": inp}]
        elif isinstance(inp, list):
            msgs = []
            for m in inp:
                c = m.get("content", "")
                if isinstance(c, list):
                    c = "".join(p.get("text", "") for p in c if isinstance(p, dict))
                msgs.append({"role": m.get("role", "user"), "content": c})
        else:
            raise ApiError("input must be a string or a list of messages")
        if body.get("instructions"):
            msgs.insert(0, {"role": "system", "content": body["instructions"]})
        prompt = template.apply(msgs)
        cfg = config_from(body, prompt, "max_output_tokens")
        text, n, reason = await run(cfg)
        rid = new_id("resp")
        return {"id": rid, "object": "response", "created_at": now(),
                "status": "completed" if reason != "length" else "incomplete", "model": cfg.model,
                "output": [{"type": "message", "id": new_id("msg"), "role": "assistant", "status": "completed",
                            "content": [{"type": "output_text", "text": text, "annotations": []}]}],
                "output_text": text, "usage": usage(dispatcher.count_tokens(prompt), n)}

    async def list_models(request: Request):
        return {"object": "list", "data": [{"id": m, "object": "model", "created": int(state["start"]),
                                            "owned_by": "air-rs"} for m in dispatcher.list_models()]}

    async def get_model(model_id: str):
        if model_id not in dispatcher.list_models():
            raise ApiError.model_not_found(model_id)
        return {"id": model_id, "object": "model", "created": int(state["start"]), "owned_by": "air-rs"}

    async def health():
        return {"status": "ok", "version": __version__, "uptime_seconds": int(time.time() - state["start"]),
                "requests_served": state["served"]}

    async def prometheus():
        eng = getattr(dispatcher, "engine", None)
        gauges = None
        if eng is not None and hasattr(eng, "stats"):
            try:      # read while the engine thread runs; a torn read only skips the gauges
                gauges = eng.stats()
            except (RuntimeError, KeyError, ValueError):
                gauges = None
        return PlainTextResponse(metrics.render(model_name, gauges), media_type="text/plain; version=0.0.4")

    for prefix in ("/v1", ""):
        app.add_api_route(prefix + "/chat/completions", chat_completions, methods=["POST"])
        app.add_api_route(prefix + "/completions", completions, methods=["POST"])
        app.add_api_route(prefix + "/embeddings", embeddings, methods=["POST"])
        app.add_api_route(prefix + "/responses", responses, methods=["POST"])
        app.add_api_route(prefix + "/models", list_models, methods=["GET"])
        app.add_api_route(prefix + "/models/{model_id}", get_model, methods=["GET"])
    app.add_api_route("/health", health, methods=["GET"])
    app.add_api_route("/metrics", prometheus, methods=["GET"])
    app.state.metrics = metrics
    app.state.dispatcher = dispatcher
    return app
