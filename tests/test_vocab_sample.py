"""Vocabulary-parallel sampling over gloo ranks against the same rule on whole logits."""
import os
import subprocess
import sys

import pytest
import torch

from air_rs.parallel.vocab_sample import sample_full
from tests.workers.vocab_sample_case import case

WORKER = os.path.join(os.path.dirname(__file__), "workers", "vocab_sample_worker.py")


def test_full_rule_greedy_ties_penalty_and_mask():
    logits, temp, top_k, top_p, counts, penalty, mask = case(203, 6)
    t, p = sample_full(logits, temp, top_k, top_p, 7, 0, counts=counts, penalty=penalty, mask=mask)
    assert int(t[0]) == 5 and float(p[0]) == 1.0                   # tie -> lowest index
    assert int(t[5]) != int(logits[5].argmax()) and int(t[5]) >= 7  # penalised, masked
    # top-k 10: always among the 10 best (temperature 0.8)
    for step in range(20):
        t, _ = sample_full(logits, temp, top_k, top_p, 7, step)
        assert int(t[1]) in torch.topk(logits[1], 10).indices.tolist()
    # same (seed, step) -> same draw; another step -> draws vary
    a = sample_full(logits, temp, top_k, top_p, 7, 3)[0]
    assert torch.equal(a, sample_full(logits, temp, top_k, top_p, 7, 3)[0])
    draws = {int(sample_full(logits, temp, top_k, top_p, 7, s)[0][4]) for s in range(30)}
    assert len(draws) > 3


def test_full_rule_matches_distribution():
    g = torch.Generator().manual_seed(1)
    logits = torch.randn(1, 12, generator=g)
    one = torch.ones(1)
    counts = torch.zeros(12)
    n = 4000
    for s in range(n):
        counts[int(sample_full(logits, one, torch.zeros(1, dtype=torch.long), one, 11, s)[0][0])] += 1
    want = torch.softmax(logits[0], 0)
    assert (counts / n - want).abs().max() < 0.03


@pytest.mark.parametrize("world,V,port", [(2, 203, 29581), (3, 301, 29582)])
def test_vocab_parallel_matches_full_logits(tmp_path, world, V, port):
    B = 6
    env = dict(os.environ, PYTHONPATH=os.getcwd())
    out = tmp_path / "o"
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr=127.0.0.1", f"--master-port={port}", WORKER, str(out), str(V), str(B)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    runs = [torch.load(f"{out}.{i}") for i in range(world)]
    logits, temp, top_k, top_p, counts, penalty, mask = case(V, B)
    for step in range(6):
        want_t, want_p = sample_full(logits, temp, top_k, top_p, 7, step, counts=counts, penalty=penalty,
                                     mask=mask)
        for rr in runs:
            got_t, got_p = rr["res"][step]
            assert torch.equal(got_t, want_t), (step, got_t, want_t)
            torch.testing.assert_close(got_p, want_p, rtol=1e-4, atol=1e-6)
    # the flat row's nucleus (0.95) is wider than 16 candidates: it takes the full-row path
    assert all(rr["fallbacks"] >= 6 for rr in runs)
    # candidates + fallbacks moved less than gathering every row's logits each step
    shard = (V + world - 1) // world
    assert runs[0]["bytes"] < 6 * B * shard * 4 * world
