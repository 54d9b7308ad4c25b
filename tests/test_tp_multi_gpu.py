"""Tensor parallelism across GPUs: fused peer-memory all-reduce vs the NCCL all-reduce.

Runs ``tests/workers/tp_worker.py`` under torch.distributed.run on 2 GPUs (skipped with
fewer). NVLS stays off so the test has no multicast objects."""
import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu


def _n_gpus():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.skipif(_n_gpus() < 2, reason="needs 2 GPUs")
def test_fused_allreduce_matches_nccl(tmp_path):
    out = tmp_path / "tp.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=os.getcwd())
    worker = os.path.join(os.path.dirname(__file__), "workers", "tp_worker.py")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29533", worker, str(out)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.loads(out.read_text())
    for pre, B in [(p, b) for p in ("", "moe_") for b in (4, 16)]:
        a, b = res[f"{pre}nccl_B{B}"], res[f"{pre}ours_B{B}"]
        # the first two tokens (prefill + first fused decode step) agree for every sequence;
        # later ones may part at fp32 summation-order near-ties of a random model
        assert all(x[:2] == y[:2] for x, y in zip(a, b)), (pre, a, b)
        same = sum(x == y for x, y in zip(a, b))
        assert same >= 0.75 * len(a), (pre, same, len(a))
        single = res[f"{pre or 'dense_'}single_B{B}"]
        # TP / EP against the unsharded model: first token from the same prefill math
        assert sum(x[:1] == y[:1] for x, y in zip(single, b)) >= 0.75 * len(b), (pre, single, b)
