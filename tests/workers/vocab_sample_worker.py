"""Vocab-parallel sampling worker: each gloo rank holds one vocabulary slice of shared
logits, samples with VocabParallelSampler and writes (tokens, probs, fallbacks, bytes)."""
import sys

import torch
import torch.distributed as dist


def main(out_path, V, B):
    from air_rs.parallel.vocab_sample import VocabParallelSampler
    dist.init_process_group("gloo")
    r, w = dist.get_rank(), dist.get_world_size()
    from tests.workers.vocab_sample_case import case
    logits, temp, top_k, top_p, counts, penalty, mask = case(V, B)
    shard = (V + w - 1) // w
    local = torch.full((B, shard), 0.0)
    part = logits[:, r * shard:(r + 1) * shard]
    local[:, : part.shape[1]] = part
    s = VocabParallelSampler(V, shard, candidates=16)
    res = []
    for step in range(6):
        t, p = s.sample(local, temp, top_k, top_p, seed=7, step=step, counts=counts, penalty=penalty, mask=mask)
        res.append((t, p))
    torch.save({"res": res, "fallbacks": s.fallbacks, "bytes": s.bytes_exchanged}, f"{out_path}.{r}")
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1], int(sys.argv[2]), int(sys.argv[3]))
