"""Analytic batch-size optimiser (reference ``src/batch_optimizer.rs``: StorageProfile /
ComputeProfile / BoptResult). Decode of a memory-bound model streams its weights once per
step, so tokens/s grows with the batch until the step becomes compute bound (or the KV
cache stops fitting). B_opt is the smallest batch at which compute time reaches the
weight-streaming time, capped by the KV capacity; streamed weights (S.L.I.P.) use the
storage/PCIe bandwidth instead of HBM.
"""
from __future__ import annotations

import math
from dataclasses import dataclass


@dataclass
class StorageProfile:
    hbm_gbs: float = 6543.0          # measured B200 copy bandwidth
    host_link_gbs: float = 55.0      # PCIe 5 x16 pinned H2D
    nvme_gbs: float = 12.0
    resident: bool = True            # weights in HBM (else streamed per step)

    def weight_gbs(self) -> float:
        return self.hbm_gbs if self.resident else min(self.host_link_gbs, self.nvme_gbs)


@dataclass
class ComputeProfile:
    tflops: float = 1657.0            # measured bf16 dense (burst)
    efficiency: float = 0.5           # achieved fraction on the decode GEMMs


@dataclass
class BoptResult:
    batch: int
    step_ms: float
    tokens_per_s: float
    bound: str                        # "memory" | "compute" | "kv"


def optimal_batch(params: float, bytes_per_param: float, kv_bytes_per_token: int, context: int,
                  free_kv_bytes: int, storage: StorageProfile | None = None,
                  compute: ComputeProfile | None = None, max_batch: int = 1024) -> BoptResult:
    storage, compute = storage or StorageProfile(), compute or ComputeProfile()
    w_s = params * bytes_per_param / (storage.weight_gbs() * 1e9)
    flop_per_tok = 2.0 * params
    peak = compute.tflops * 1e12 * compute.efficiency
    b_compute = max(1, math.ceil(w_s * peak / flop_per_tok))
    b_kv = max(1, free_kv_bytes // max(1, kv_bytes_per_token * context))
    b = min(b_compute, b_kv, max_batch)
    kv_s = b * kv_bytes_per_token * context / (storage.hbm_gbs * 1e9)
    step = max(w_s + kv_s, b * flop_per_tok / peak)
    bound = "kv" if b == b_kv and b_kv < b_compute else ("compute" if b == b_compute else "memory")
    return BoptResult(b, step * 1e3, b / step, bound)
