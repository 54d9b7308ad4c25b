"""Failure detection without any GPU fault: host-injected rank failures on gloo ranks, a
failing engine step in the server, and PD transfer timeouts (test_pd.py)."""
import json
import os
import subprocess
import sys

import pytest

WORKER = os.path.join(os.path.dirname(__file__), "workers", "health_worker.py")


def _launch(mode, out, port):
    env = dict(os.environ, PYTHONPATH=os.getcwd(), MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
               WORLD_SIZE="3")
    procs = [subprocess.Popen([sys.executable, WORKER, mode, str(out)], env=dict(env, RANK=str(r), LOCAL_RANK=str(r)),
                              stdout=subprocess.PIPE, stderr=subprocess.PIPE) for r in range(3)]
    for p in procs:
        try:
            p.wait(timeout=60)
        except subprocess.TimeoutExpired:
            p.kill()
            raise
    return json.loads(out.read_text())


def test_heartbeat_detects_hung_and_exited_ranks(tmp_path):
    res = _launch("heartbeat", tmp_path / "hb.json", 29571)
    assert res["dead"] == [1, 2] and res["raised"] and res["elapsed"] < 3.0


def test_process_group_timeout_ends_collective_with_dead_rank(tmp_path):
    res = _launch("pgtimeout", tmp_path / "pg.json", 29572)
    assert res["error"] is not None and res["elapsed"] < 30.0


def test_server_fails_requests_on_engine_error_and_keeps_serving():
    import asyncio
    from air_rs.serve.dispatcher import EngineDispatcher, GenerateConfig
    from air_rs.runtime.engine import Engine
    from air_rs.models.config import tiny_llama
    from air_rs.tokenizer import Tokenizer

    class Broken(Engine):
        def step(self):
            if getattr(self, "_fail", True):
                self._fail = False
                raise RuntimeError("device kernel reported error code 2 (peer timeout)")
            return super().step()

    cfg = tiny_llama()
    from air_rs.models.random_init import random_tensors
    from air_rs.models.reference import OracleModel
    from air_rs.gguf import GGMLType
    recs = list(random_tensors(cfg, GGMLType.Q8_0, seed=0, device="cpu"))
    eng = Broken(cfg, None, Tokenizer.byte_vocab(cfg.vocab_size, 1, 2),
                 oracle=OracleModel(cfg, {n: (r, q, s) for n, r, q, s in recs}))
    d = EngineDispatcher(eng, "m")

    async def collect(prompt):
        chunks = []
        async for c in d.generate(GenerateConfig(prompt=prompt, max_tokens=3, temperature=0.0)):
            chunks.append(c)
        return chunks

    try:
        first = asyncio.run(collect("hello"))
        assert first[-1].is_stop and first[-1].error and "peer timeout" in first[-1].error
        second = asyncio.run(collect("again"))
        assert second[-1].is_stop and not second[-1].error and len(second) == 4
        assert d.errors == 1 and not eng.running and not eng.waiting
    finally:
        d.shutdown()


def test_multi_rank_serving_mirrors_rank0(tmp_path):
    """serve --tp N design on gloo ranks: rank 0 answers concurrent HTTP requests, the
    follower mirrors every admission and step, and both generate the same tokens."""
    import json
    import subprocess
    import sys
    out = tmp_path / "serve"
    worker = os.path.join(os.path.dirname(__file__), "workers", "serve_worker.py")
    env = dict(os.environ, PYTHONPATH=os.getcwd())
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29597", worker, str(out)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    r0 = json.loads(open(f"{out}.0").read())
    r1 = json.loads(open(f"{out}.1").read())
    assert r0["embed_ok"]
    assert all(code == 200 and n == 5 + int(i) for i, (code, _, n) in r0["texts"].items()), r0["texts"]
    assert len(r0["history"]) == 4 and r0["history"] == r1["history"]
    assert r0["ticks"] == r1["ticks"]
