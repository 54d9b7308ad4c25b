"""Worker of the pipeline-parallel tests (torch.distributed.run).

Mode "fake" (gloo, CPU): stages are affine maps, so the pipelined result can be checked
exactly. Mode "model" (NCCL, one GPU per stage): a random model split by layers; rank 0
writes the generated tokens to the output file."""
import json
import os
import sys

import torch
import torch.distributed as dist

from air_rs.parallel.pp import MicroBatch, PipelineRunner


class FakeStage:
    def __init__(self, rank, world):
        self.rank, self.world = rank, world
        self.first, self.last = rank == 0, rank == world - 1

    def forward(self, mb, h):
        x = mb.ids.float()[:, None].repeat(1, 4) if h is None else h
        y = x * 2 + self.rank
        if self.last:
            return y.sum(1)[mb.last_rows].to(torch.int32)
        return y


def fake(out_path):
    dist.init_process_group("gloo")
    r, w = dist.get_rank(), dist.get_world_size()
    pr = PipelineRunner(FakeStage(r, w), r, w, 4, "cpu")
    mbs = []
    for m in range(3):
        ids = torch.arange(m, m + 5, dtype=torch.int32)
        z = torch.zeros(5, dtype=torch.int32)
        mbs.append(MicroBatch(ids, z, z.long(), z, torch.zeros(1, 1, dtype=torch.int32),
                              torch.tensor([4, 2]), torch.zeros(2, dtype=torch.int32)))
    res = [t.tolist() for t in pr.run(mbs)]
    if r == 0:
        json.dump(res, open(out_path, "w"))
    dist.barrier()
    dist.destroy_process_group()


def model(out_path):
    from air_rs.gguf import GGMLType
    from air_rs.models.config import ModelConfig
    from air_rs.models.random_init import random_tensors
    from air_rs.parallel.pp import PipelineEngine, partition_layers
    from air_rs.runtime.builder import build_runner
    dist.init_process_group("nccl")
    r, w = dist.get_rank(), dist.get_world_size()
    torch.cuda.set_device(r)
    cfg = ModelConfig(n_layers=4, n_heads=8, n_kv_heads=2, hidden_dim=1024, intermediate_dim=2816,
                      vocab_size=4096, head_dim=128)
    recs = list(random_tensors(cfg, GGMLType.Q4_K, seed=0, device="cpu"))
    rng = partition_layers(cfg.n_layers, w)[r]
    rn = build_runner(cfg, iter(recs), device=f"cuda:{r}", max_batch=8, max_model_len=256, num_blocks=64,
                      layer_range=rng)
    eng = PipelineEngine(rn, r, w, micro_batches=2, bos=cfg.bos_token_id)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, cfg.vocab_size, (int(n),), generator=g).tolist() for n in (17, 30, 9)]
    outs = eng.generate(prompts, 12)
    if r == 0:
        json.dump({"outs": outs, "prompts": prompts, "sent": eng.pipe.sent_bytes}, open(out_path, "w"))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    {"fake": fake, "model": model}[sys.argv[1]](sys.argv[2])
