"""Ring attention worker: each gloo rank holds one chunk of a prompt; writes its output."""
import json
import sys

import torch
import torch.distributed as dist


def main(out_path, n_tokens, causal):
    from air_rs.parallel.cp import ring_attention, split_sequence
    dist.init_process_group("gloo")
    r, w = dist.get_rank(), dist.get_world_size()
    g = torch.Generator().manual_seed(0)
    q = torch.randn(n_tokens, 4, 16, generator=g)
    k = torch.randn(n_tokens, 2, 16, generator=g)
    v = torch.randn(n_tokens, 2, 16, generator=g)
    chunks = split_sequence(n_tokens, w)
    s, e = chunks[r]
    out = ring_attention(q[s:e], k[s:e], v[s:e], s, [c[0] for c in chunks], causal=causal)
    torch.save(out, f"{out_path}.{r}")
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1], int(sys.argv[2]), sys.argv[3] == "1")
