"""Worker of the multi-GPU tensor-parallel test (launched by torch.distributed.run).

Builds the same random model with the NCCL all-reduce and with the fused peer-memory
all-reduce, decodes greedily with both, and writes the tokens and timings to a JSON file
(rank 0) for the test to check."""
import json
import os
import sys
import time

import torch

from air_rs.models.config import ModelConfig
from air_rs.parallel.symm import maybe_fused_tp
from air_rs.parallel.tp import init_from_env
from air_rs.runtime.builder import random_engine
from air_rs.runtime.engine import SamplingParams


def main(out_path: str):
    tp0 = init_from_env("nccl")
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    cfg = ModelConfig(n_layers=4, n_heads=16, n_kv_heads=8, hidden_dim=2048, intermediate_dim=4096,
                      vocab_size=4096, rope_theta=10000.0, rms_norm_eps=1e-5, head_dim=128,
                      bos_token_id=1, eos_token_id=2)
    g = torch.Generator().manual_seed(7)
    res = {"world": tp0.world_size}
    moe = ModelConfig(n_layers=2, n_heads=8, n_kv_heads=4, hidden_dim=1024, intermediate_dim=1024,
                      vocab_size=4096, rope_theta=10000.0, rms_norm_eps=1e-5, head_dim=128,
                      bos_token_id=1, eos_token_id=2, n_experts=4, moe_top_k=2)
    for name, mcfg in (("dense", cfg), ("moe", moe)):
        if name == "moe":
            cfg = mcfg
        run_model(res, name, cfg, tp0, dev, g)
    if tp0.rank == 0:
        with open(out_path, "w") as f:
            json.dump(res, f)
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()


def run_model(res, name, cfg, tp0, dev, g):
    for B in (4, 16):
        prompts = [torch.randint(3, cfg.vocab_size, (int(l),), generator=g).tolist()
                   for l in torch.randint(5, 40, (B,), generator=g)]
        for impl in ("nccl", "ours"):
            tp = maybe_fused_tp(tp0, impl=impl, max_rows=B, hidden=cfg.hidden_dim, device=dev)
            eng = random_engine(cfg, seed=3, device=dev, max_batch=B, max_model_len=256, tp=tp)
            sp = SamplingParams(max_tokens=12, temperature=0.0, repetition_penalty=1.0, ignore_eos=True)
            out = eng.generate_ids(prompts, sp)
            eng.runner.check_errors()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            eng.generate_ids(prompts, sp)
            torch.cuda.synchronize()
            key = f"{impl}_B{B}" if name == "dense" else f"{name}_{impl}_B{B}"
            res[key] = out
            res[key + "_s"] = time.perf_counter() - t0
            if impl == "ours":
                tp.peer.close()
            del eng
            torch.cuda.empty_cache()
        if tp0.rank == 0:     # the same model on one GPU (no TP / EP)
            eng = random_engine(cfg, seed=3, device=dev, max_batch=B, max_model_len=256)
            res[f"{name}_single_B{B}"] = eng.generate_ids(prompts, sp)
            del eng
            torch.cuda.empty_cache()


if __name__ == "__main__":
    main(sys.argv[1])
