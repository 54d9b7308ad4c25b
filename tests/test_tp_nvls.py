"""Tensor parallelism with the NVLink SHARP all-reduce (multimem.ld_reduce over a
multicast-bound symmetric buffer, fused with the following norm) vs the NCCL all-reduce,
compared on the logits of every decode step at 2 GPUs (4 and 8 when present). Skipped when
the GPUs offer no multicast object."""
import os
import subprocess
import sys

import pytest
import torch

from test_tp_multi_gpu import _compare

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_nvls_logits_match_nccl(tmp_path, world):
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    if n < world:
        pytest.skip(f"needs {world} GPUs")
    out = tmp_path / "nvls.pt"
    env = dict(os.environ, PYTHONPATH=os.getcwd())
    worker = os.path.join(os.path.dirname(__file__), "workers", "tp_nvls_worker.py")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr=127.0.0.1", f"--master-port={29633 + world}", worker, str(out)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    if r.returncode != 0 and "no multicast object" in (r.stdout + r.stderr):
        pytest.skip("no NVLS multicast on these GPUs")
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = torch.load(out, weights_only=False)
    report = {f"B{B}": _compare(res[f"nvls_B{B}"], res[f"nccl_B{B}"], 2e-2) for B in (4, 16)}
    print(report)
    assert all(v <= 2e-2 for v in report.values()), report
