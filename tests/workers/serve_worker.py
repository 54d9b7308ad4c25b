"""Worker of the multi-rank serving test: gloo ranks on the CPU, each with the same
random tiny model on the CPU oracle engine. Rank 0 serves HTTP (FastAPI TestClient) to
several concurrent clients through ``DistributedDispatcher``; the other ranks mirror its
engine loop with ``serve_follower``. Every rank writes what it generated to argv[1].<rank>."""
import json
import os
import sys
import threading
from datetime import timedelta

import torch
import torch.distributed as dist


def build_engine():
    from air_rs.gguf import GGMLType
    from air_rs.models.config import tiny_llama
    from air_rs.models.random_init import random_tensors
    from air_rs.models.reference import OracleModel
    from air_rs.runtime.engine import Engine
    from air_rs.tokenizer import Tokenizer
    cfg = tiny_llama()
    recs = list(random_tensors(cfg, GGMLType.Q8_0, seed=0, device="cpu"))
    return Engine(cfg, None, Tokenizer.byte_vocab(cfg.vocab_size, 1, 2),
                  oracle=OracleModel(cfg, {n: (r, q, s) for n, r, q, s in recs}))


def main(out):
    dist.init_process_group("gloo", timeout=timedelta(seconds=60))
    rank = dist.get_rank()
    torch.set_num_threads(1)
    from air_rs.serve.distributed import DistributedDispatcher
    eng = build_engine()
    d = DistributedDispatcher(eng, "tiny", idle_tick_s=0.2)
    res = {"rank": rank}
    if rank == 0:
        from fastapi.testclient import TestClient
        from air_rs.serve.app import create_app
        client = TestClient(create_app(d, "tiny"))
        texts = {}

        def call(i):
            r = client.post("/v1/completions", json={"prompt": f"request {i} " * (i + 1), "max_tokens": 5 + i,
                                                     "temperature": 0.0})
            texts[i] = (r.status_code, r.json()["choices"][0]["text"], r.json()["usage"]["completion_tokens"])

        ths = [threading.Thread(target=call, args=(i,)) for i in range(4)]
        for t in ths:
            t.start()
        for t in ths:
            t.join()
        e = client.post("/v1/embeddings", json={"input": "abc"})
        res["embed_ok"] = e.status_code == 200
        res["texts"] = texts
        d.shutdown()
    else:
        d.serve_follower()
    res["history"] = {str(k): v for k, v in d.history.items()}
    res["ticks"] = d.ticks
    with open(f"{out}.{rank}", "w") as f:
        json.dump(res, f)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
