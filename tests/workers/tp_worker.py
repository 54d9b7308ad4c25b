"""Worker of the multi-GPU tensor-parallel test (launched by torch.distributed.run).

Builds the same random model three ways: unsharded on one GPU (rank 0), tensor-parallel
with the NCCL all-reduce, and tensor-parallel with the fused peer-memory all-reduce. Each
decodes the same prompts greedily; after every decode step the full-vocabulary logits of
every row are kept. Rank 0 saves tokens and logits (torch.save) for the test to compare."""
import os
import sys

import torch

from air_rs.models.config import ModelConfig
from air_rs.parallel.symm import maybe_fused_tp
from air_rs.parallel.tp import init_from_env
from air_rs.runtime.builder import random_engine
from air_rs.runtime.engine import SamplingParams

STEPS = 10


def decode_with_logits(eng, prompts, sp):
    """Greedy decode; returns (tokens per prompt, [steps, B, V] logits of each decode step)."""
    rids = [eng.add_request(p, sp) for p in prompts]
    rn = eng.runner
    logits = []
    while eng.has_unfinished():
        batch = [r for r in eng.running if r.output_ids and not r.finished]
        eng.step()
        if batch or eng.running:
            n = len(prompts)
            logits.append(rn.logits_full[:n, : eng.cfg.vocab_size].float().cpu().clone())
    eng.runner.check_errors()
    return [eng.finished[r].output_ids for r in rids], torch.stack(logits)


def main(out_path: str):
    tp0 = init_from_env("nccl")
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    dense = ModelConfig(n_layers=4, n_heads=16, n_kv_heads=8, hidden_dim=2048, intermediate_dim=4096,
                        vocab_size=4096, rope_theta=10000.0, rms_norm_eps=1e-5, head_dim=128,
                        bos_token_id=1, eos_token_id=2)
    moe = ModelConfig(n_layers=2, n_heads=16, n_kv_heads=8, hidden_dim=2048, intermediate_dim=1024,
                      vocab_size=4096, rope_theta=10000.0, rms_norm_eps=1e-5, head_dim=128,
                      bos_token_id=1, eos_token_id=2, n_experts=8, moe_top_k=2)
    g = torch.Generator().manual_seed(7)
    res = {"world": tp0.world_size}
    for name, cfg in (("dense", dense), ("moe", moe)):
        for B in (4, 16):
            prompts = [torch.randint(3, cfg.vocab_size, (int(l),), generator=g).tolist()
                       for l in torch.randint(5, 40, (B,), generator=g)]
            sp = SamplingParams(max_tokens=STEPS, temperature=0.0, repetition_penalty=1.0, ignore_eos=True)
            for impl in ("nccl", "ours", "ours_vg"):
                # ours_vg: the vocabulary-parallel greedy head (per-rank argmax partials are
                # gathered, not the logits): tokens only
                os.environ["AIR_VOCAB_GREEDY"] = "1" if impl == "ours_vg" else "0"
                tp = maybe_fused_tp(tp0, impl="nccl" if impl == "nccl" else "ours", max_rows=B,
                                    hidden=cfg.hidden_dim, device=dev)
                eng = random_engine(cfg, seed=3, device=dev, max_batch=B, max_model_len=256, tp=tp)
                eng.runner.gemv_max_b = 8         # B=4: the GEMV chain; B=16: the GEMM step
                if impl == "ours_vg":
                    assert eng.runner.vocab_greedy
                    rids = [eng.add_request(p, sp) for p in prompts]
                    while eng.has_unfinished():
                        eng.step()
                    eng.runner.check_errors()
                    res[f"{name}_{impl}_B{B}"] = [eng.finished[r].output_ids for r in rids]
                else:
                    res[f"{name}_{impl}_B{B}"] = decode_with_logits(eng, prompts, sp)
                os.environ.pop("AIR_VOCAB_GREEDY", None)
                torch.cuda.synchronize()
                torch.distributed.barrier()
                eng.runner.graphs.clear()
                if impl != "nccl":
                    tp.peer.close()
                del eng
                torch.cuda.empty_cache()
            if tp0.rank == 0:     # the same model on one GPU (no TP / EP)
                eng = random_engine(cfg, seed=3, device=dev, max_batch=B, max_model_len=256)
                eng.runner.gemv_max_b = 8
                res[f"{name}_single_B{B}"] = decode_with_logits(eng, prompts, sp)
                del eng
                torch.cuda.empty_cache()
            torch.distributed.barrier()
    if tp0.rank == 0:
        torch.save(res, out_path)
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
