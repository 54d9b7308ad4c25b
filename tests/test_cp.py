"""Context-parallel ring attention over gloo ranks against dense attention."""
import os
import subprocess
import sys

import pytest
import torch

from air_rs.models.reference import attention_reference
from air_rs.parallel.cp import split_sequence

WORKER = os.path.join(os.path.dirname(__file__), "workers", "cp_worker.py")


def test_split_sequence():
    assert split_sequence(10, 3) == [(0, 4), (4, 7), (7, 10)]
    assert split_sequence(2, 3) == [(0, 1), (1, 2), (2, 2)]


@pytest.mark.parametrize("world,n,causal,port", [(2, 37, True, 29571), (3, 50, True, 29572), (3, 20, False, 29573),
                                                 (3, 2, True, 29574)])
def test_ring_attention_matches_dense(tmp_path, world, n, causal, port):
    env = dict(os.environ, PYTHONPATH=os.getcwd())
    out = tmp_path / "o"
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr=127.0.0.1", f"--master-port={port}", WORKER, str(out), str(n), "1" if causal else "0"]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    got = torch.cat([torch.load(f"{out}.{i}") for i in range(world)], 0)
    g = torch.Generator().manual_seed(0)
    q = torch.randn(n, 4, 16, generator=g)
    k = torch.randn(n, 2, 16, generator=g)
    v = torch.randn(n, 2, 16, generator=g)
    ref = attention_reference(q, k, v, causal=causal)
    torch.testing.assert_close(got, ref, rtol=1e-4, atol=1e-5)
