"""Worker of the NVLS tensor-parallel test (launched by torch.distributed.run).

Decodes the same prompts greedily with the NCCL all-reduce and with the NVLink SHARP
(multimem.ld_reduce) all-reduce, keeping the full-vocabulary logits of every decode step.
Every rank synchronises and meets at a barrier before the symmetric buffer is released, so
no rank leaves while a multicast object it is bound to is still in use. Rank 0 saves the
results (torch.save) for the test to compare."""
import os
import sys

import torch

from air_rs.models.config import ModelConfig
from air_rs.parallel.symm import maybe_fused_tp
from air_rs.parallel.tp import init_from_env
from air_rs.runtime.builder import random_engine
from air_rs.runtime.engine import SamplingParams

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from tp_worker import decode_with_logits  # noqa: E402


def main(out_path: str):
    tp0 = init_from_env("nccl")
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    cfg = ModelConfig(n_layers=4, n_heads=16, n_kv_heads=8, hidden_dim=2048, intermediate_dim=4096,
                      vocab_size=4096, rope_theta=10000.0, rms_norm_eps=1e-5, head_dim=128,
                      bos_token_id=1, eos_token_id=2)
    g = torch.Generator().manual_seed(11)
    res = {"world": tp0.world_size}
    for B in (4, 16):
        prompts = [torch.randint(3, cfg.vocab_size, (int(l),), generator=g).tolist()
                   for l in torch.randint(5, 40, (B,), generator=g)]
        sp = SamplingParams(max_tokens=10, temperature=0.0, repetition_penalty=1.0, ignore_eos=True)
        for impl in ("nccl", "nvls"):
            tp = maybe_fused_tp(tp0, impl=impl, max_rows=B, hidden=cfg.hidden_dim, device=dev)
            eng = random_engine(cfg, seed=3, device=dev, max_batch=B, max_model_len=256, tp=tp)
            eng.runner.gemv_max_b = 8         # B=4: the GEMV path; B=16: the GEMM step
            res[f"{impl}_B{B}"] = decode_with_logits(eng, prompts, sp)
            torch.cuda.synchronize()
            torch.distributed.barrier()
            eng.runner.graphs.clear()
            if impl == "nvls":
                tp.peer.check()
                torch.cuda.synchronize()
                torch.distributed.barrier()
                tp.peer.close()
            del eng
            torch.cuda.empty_cache()
            torch.distributed.barrier()
    if tp0.rank == 0:
        torch.save(res, out_path)
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
