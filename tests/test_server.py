"""REST server: routes, SSE streaming, error envelope, auth, rate limit, metrics (CPU)."""
import json

import pytest
from fastapi.testclient import TestClient

from air_rs.serve.app import create_app
from air_rs.serve.dispatcher import EngineDispatcher, MockDispatcher
from air_rs.serve.openai import LatencyHistogram, RateLimiter


@pytest.fixture()
def client():
    return TestClient(create_app(MockDispatcher("mock"), "mock"))


def test_chat_completion(client):
    r = client.post("/v1/chat/completions", json={"model": "mock", "messages": [{"role": "user", "content": "hi"}]})
    assert r.status_code == 200
    body = r.json()
    assert body["object"] == "chat.completion"
    assert body["choices"][0]["message"]["content"] == "Hello, world!"
    assert body["choices"][0]["finish_reason"] == "stop"
    assert body["usage"]["completion_tokens"] == 4


def test_chat_stream_sse(client):
    with client.stream("POST", "/chat/completions",
                       json={"messages": [{"role": "user", "content": "hi"}], "stream": True}) as r:
        lines = [l for l in r.iter_lines() if l.startswith("data: ")]
    assert lines[-1] == "data: [DONE]"
    chunks = [json.loads(l[6:]) for l in lines[:-1]]
    assert chunks[0]["choices"][0]["delta"]["role"] == "assistant"
    assert "".join(c["choices"][0]["delta"].get("content", "") for c in chunks) == "Hello, world!"
    assert chunks[-1]["choices"][0]["finish_reason"] == "stop"


def test_completions_length_and_models(client):
    r = client.post("/v1/completions", json={"prompt": "x", "max_tokens": 2})
    assert r.json()["choices"][0]["finish_reason"] == "length"
    assert r.json()["choices"][0]["text"] == "Hello,"
    assert client.get("/v1/models").json()["data"][0]["id"] == "mock"
    assert client.get("/models/mock").status_code == 200
    r = client.get("/v1/models/nope")
    assert r.status_code == 404 and r.json()["error"]["code"] == "model_not_found"


def test_errors_envelope(client):
    r = client.post("/v1/chat/completions", json={"messages": []})
    assert r.status_code == 400 and r.json()["error"]["type"] == "invalid_request_error"
    r = client.post("/v1/completions", json={"prompt": "x", "temperature": 9})
    assert r.status_code == 400
    r = client.post("/v1/chat/completions", json={"model": "other", "messages": [{"role": "user", "content": "x"}]})
    assert r.status_code == 404


def test_embeddings_responses_health_metrics(client):
    r = client.post("/v1/embeddings", json={"input": ["ab", "abc"]})
    assert [d["embedding"][0] for d in r.json()["data"]] == [2.0, 3.0]
    r = client.post("/v1/responses", json={"input": "hi", "instructions": "be nice"})
    assert r.json()["output_text"] == "Hello, world!" and r.json()["status"] == "completed"
    h = client.get("/health").json()
    assert h["status"] == "ok" and h["requests_served"] >= 1
    m = client.get("/metrics").text
    assert "air_requests_total" in m and "air_ttft_ms_bucket" in m


def test_metrics_export_engine_gauges():
    from air_rs.serve.openai import PrometheusMetrics
    text = PrometheusMetrics().render("m", {"kv_utilization": 0.25, "running": 3, "flag": True, "name": "x"})
    assert 'air_kv_utilization{model="m"} 0.25' in text and 'air_running{model="m"} 3' in text
    assert "air_flag" not in text and "air_name" not in text


def test_auth_and_rate_limit():
    c = TestClient(create_app(MockDispatcher("mock"), "mock", api_keys=["sk-1"], rate_limit=(0.0001, 2)))
    body = {"prompt": "x"}
    assert c.post("/v1/completions", json=body).status_code == 401
    hdr = {"Authorization": "Bearer sk-1"}
    assert c.post("/v1/completions", json=body, headers=hdr).status_code == 200
    assert c.post("/v1/completions", json=body, headers=hdr).status_code == 200
    assert c.post("/v1/completions", json=body, headers=hdr).status_code == 429


def test_rate_limiter_refill_and_histogram():
    rl = RateLimiter(rate=1.0, burst=1)
    assert rl.allow("a", 0.0) and not rl.allow("a", 0.5) and rl.allow("a", 1.6)
    h = LatencyHistogram()
    for v in range(1, 101):
        h.record(float(v))
    assert h.percentile(50) == 50.0 and h.percentile(99) == 99.0


def test_engine_dispatcher_cpu(tmp_path):
    from air_rs.gguf import GGMLType
    from air_rs.models.config import tiny_llama
    from air_rs.models.random_init import write_random_gguf
    from air_rs.runtime.builder import engine_from_gguf
    p = write_random_gguf(str(tmp_path / "t.gguf"), tiny_llama(), GGMLType.Q8_0)
    d = EngineDispatcher(engine_from_gguf(p, device="cpu"), "tiny")
    try:
        c = TestClient(create_app(d, "tiny"))
        r = c.post("/v1/completions", json={"prompt": "ab", "max_tokens": 4, "temperature": 0})
        assert r.status_code == 200 and r.json()["usage"]["completion_tokens"] >= 1
        e = c.post("/v1/embeddings", json={"input": "abc"}).json()["data"][0]["embedding"]
        assert len(e) == 256
    finally:
        d.shutdown()


def test_replica_router_balances_and_skips_failed_replica():
    """Data-parallel replicas: least-in-flight routing with round robin on ties, and a
    replica that raises before streaming is skipped for the next one."""
    import asyncio
    from air_rs.serve.dispatcher import GenerateConfig, TokenChunk
    from air_rs.serve.replicas import ReplicaRouter

    class Slow(MockDispatcher):
        async def generate(self, config):
            await asyncio.sleep(0.01)
            async for c in super().generate(config):
                yield c

    class Broken(MockDispatcher):
        async def generate(self, config):
            raise RuntimeError("GPU lost")
            yield

    reps = [Slow("m", ["a"]), Slow("m", ["b"]), Slow("m", ["c"])]
    router = ReplicaRouter(reps, "m")

    async def one(i):
        return [c async for c in router.generate(GenerateConfig(prompt=str(i), max_tokens=4))]

    async def many():
        return await asyncio.gather(*(one(i) for i in range(6)))

    outs = asyncio.run(many())
    assert sorted(o[0].text for o in outs) == ["a", "a", "b", "b", "c", "c"]
    assert router.served == [2, 2, 2] and router.in_flight == [0, 0, 0]
    r2 = ReplicaRouter([Broken("m"), MockDispatcher("m", ["ok"])], "m")
    for _ in range(3):
        out = asyncio.run(_collect(r2))
        assert out[0].text == "ok" and out[-1].finish_reason == "stop"
    dead = ReplicaRouter([Broken("m")], "m")
    assert asyncio.run(_collect(dead))[-1].error.startswith("all replicas failed")
    client = TestClient(create_app(ReplicaRouter([MockDispatcher("m"), MockDispatcher("m")], "m"), "m"))
    r = client.post("/v1/completions", json={"prompt": "x", "max_tokens": 8})
    assert r.json()["choices"][0]["text"] == "Hello, world!"


async def _collect(router):
    from air_rs.serve.dispatcher import GenerateConfig
    return [c async for c in router.generate(GenerateConfig(prompt="p", max_tokens=4))]
