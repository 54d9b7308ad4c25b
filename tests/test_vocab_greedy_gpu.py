"""Vocabulary-parallel greedy sampling kernels (the TP decode head): W shards of one logit
matrix processed as W ranks would (partial pass with the shard's global offset, partials laid
out [W, B, chunks] as an all-gather leaves them, merge) give the whole-vocabulary sampler's
tokens, with repetition penalty, grammar mask, ties and a padded last shard."""
import pytest
import torch

from air_rs import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("W", [2, 3, 8])
def test_vocab_parallel_greedy_matches_full_sampler(W):
    B, V = 5, 128256
    g = torch.Generator().manual_seed(W)
    logits = torch.randn(B, V, generator=g)
    top = logits.argmax(-1)
    logits[3, 77] = logits[3, 100000] = logits[3].max() + 1.0     # tie: lowest index wins
    counts = torch.zeros(8, V, dtype=torch.uint8)
    counts[1, top[1]] = 4                                           # penalise row 1's argmax
    count_row = torch.tensor([0, 1, 2, 3, 4], dtype=torch.int32)
    mask = torch.full((B, (V + 31) // 32), -1, dtype=torch.int32)
    w_, b_ = int(top[2]) // 32, int(top[2]) % 32                   # forbid row 2's argmax
    m = (0xFFFFFFFF & ~(1 << b_))
    mask[2, w_] = m - (1 << 32) if m >= 1 << 31 else m
    pen = torch.full((B,), 1.2)
    want = torch.zeros(B, dtype=torch.int32, device=DEV)
    ops.sample(logits.to(DEV), want, counts=counts.to(DEV), count_row=count_row.to(DEV), mask=mask.to(DEV),
               temperature=torch.zeros(B, device=DEV), penalty=pen.to(DEV))
    per = -(-V // W)
    per = -(-per // 32) * 32                     # shard width (multiple of 32; last shard padded)
    nch = ops.sampler_chunks(per)
    allp = torch.zeros(W * B * nch * 4, device=DEV)
    full = torch.zeros(B, W * per)
    full[:, :V] = logits
    full[:, V:] = 1e4                             # padding columns must never win
    for r in range(W):
        shard = full[:, r * per:(r + 1) * per].contiguous().to(DEV)
        valid = max(0, min(per, V - r * per))
        ops.sample_partial(shard, allp[r * B * nch * 4:(r + 1) * B * nch * 4], v_off=r * per, V_total=V,
                           counts=counts.to(DEV), count_row=count_row.to(DEV), mask=mask.to(DEV),
                           penalty=pen.to(DEV), B=B, V=valid, nch=nch)
    got = torch.zeros(B, dtype=torch.int32, device=DEV)
    step = torch.zeros(1, dtype=torch.int64, device=DEV)
    ops.sample_greedy_merge(allp, got, W=W, B=B, nch=nch, step=step)
    torch.cuda.synchronize()
    assert got.cpu().tolist() == want.cpu().tolist()
    assert int(got[3]) == 77 and int(step) == 1
    assert int(got[1]) != int(top[1]) and int(got[2]) != int(top[2])
