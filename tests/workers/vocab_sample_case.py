"""Shared inputs of the vocab-parallel sampling test (rows: greedy, top-k, nucleus that fits
in the candidates, wide nucleus, whole-vocabulary draw, masked + penalised greedy)."""
import torch


def case(V, B):
    g = torch.Generator().manual_seed(0)
    logits = torch.randn(B, V, generator=g) * 3
    logits[3] = torch.randn(V, generator=g) * 0.05          # flat row: nucleus wider than C
    logits[0, 5] = logits[0, V - 3] = logits[0].max() + 1    # greedy tie: lowest index wins
    temp = torch.tensor([0.0, 0.8, 1.0, 1.0, 1.2, 0.0][:B])
    top_k = torch.tensor([0, 10, 0, 0, 0, 0][:B])
    top_p = torch.tensor([1.0, 0.9, 0.5, 0.95, 1.0, 1.0][:B])
    counts = torch.zeros(B, V, dtype=torch.int32)
    counts[5, logits[5].argmax()] = 2                         # penalised away from the argmax
    penalty = torch.tensor([1.0, 1.0, 1.0, 1.0, 1.0, 100.0][:B])
    mask = torch.ones(B, V, dtype=torch.bool)
    mask[5, :7] = False
    return logits, temp, top_k, top_p, counts, penalty, mask
