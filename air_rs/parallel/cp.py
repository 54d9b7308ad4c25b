"""Context-parallel (ring) attention for long prompts (the reference has single-device blockwise
attention only, ``src/chunked_attn.rs``, described as "ring-compatible").

The prompt is split into contiguous chunks, one per rank. Each rank keeps its queries and
passes its K/V chunk around the ring: at every hop a rank attends its queries to the K/V chunk
it holds (with the causal rule on global positions), folds the result into a running
(max, sum, output) online softmax, and forwards the chunk to the next rank while receiving the
previous rank's — non-blocking send/recv, so the transfer of hop h+1 overlaps the math of hop
h. After world-1 hops every query has seen every key it may see. Works over NCCL (GPU
tensors) or gloo (CPU tensors).
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist


def _block(q, k, v, q_pos, k_pos, causal: bool, scale: float):
    """Scores of q [Sq, H, D] against one K/V chunk [Sk, Hkv, D] -> (m, l, o) per query row."""
    rep = q.shape[1] // k.shape[1]
    kk = k.float().repeat_interleave(rep, 1)
    vv = v.float().repeat_interleave(rep, 1)
    s = torch.einsum("shd,thd->hst", q.float(), kk) * scale
    if causal:
        s = s.masked_fill(~(k_pos[None, :] <= q_pos[:, None])[None], float("-inf"))
    m = s.amax(-1)                                     # [H, Sq]
    safe = torch.where(torch.isinf(m), torch.zeros_like(m), m)
    p = torch.exp(s - safe[..., None])
    return m, p.sum(-1), torch.einsum("hst,thd->hsd", p, vv)


def ring_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_offset: int, kv_offsets: list[int],
                   causal: bool = True, group=None) -> torch.Tensor:
    """q [Sq, H, D] of this rank's chunk starting at global position ``q_offset``; k / v
    [Sk, Hkv, D] this rank's K/V chunk; ``kv_offsets[r]`` the global start of rank r's chunk
    (chunks may differ in length). Returns this rank's attention output [Sq, H, D]."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    D = q.shape[-1]
    scale = 1.0 / math.sqrt(D)
    q_pos = torch.arange(q_offset, q_offset + q.shape[0], device=q.device)
    H, Sq = q.shape[1], q.shape[0]
    M = torch.full((H, Sq), float("-inf"), device=q.device)
    L = torch.zeros(H, Sq, device=q.device)
    O = torch.zeros(H, Sq, D, device=q.device)
    lens = torch.zeros(world, dtype=torch.long, device=k.device)
    lens[rank] = k.shape[0]
    dist.all_reduce(lens, group=group)
    cur_k, cur_v, src = k.contiguous(), v.contiguous(), rank
    nxt, prv = (rank + 1) % world, (rank - 1) % world
    g = lambda r: dist.get_global_rank(group, r) if group is not None else r
    for hop in range(world):
        reqs = []
        if hop < world - 1:
            src_next = (src - 1) % world
            n = int(lens[src_next])
            rk = torch.empty((n,) + tuple(k.shape[1:]), dtype=k.dtype, device=k.device)
            rv = torch.empty_like(rk)
            reqs = [dist.isend(cur_k, g(nxt), group=group), dist.isend(cur_v, g(nxt), group=group),
                    dist.irecv(rk, g(prv), group=group), dist.irecv(rv, g(prv), group=group)]
        k_pos = torch.arange(kv_offsets[src], kv_offsets[src] + cur_k.shape[0], device=q.device)
        if cur_k.shape[0]:
            m, l, o = _block(q, cur_k, cur_v, q_pos, k_pos, causal, scale)
            M_new = torch.maximum(M, m)
            safe = torch.where(torch.isinf(M_new), torch.zeros_like(M_new), M_new)
            a, b = torch.exp(M - safe), torch.exp(m - safe)
            L = L * a + l * b
            O = O * a[..., None] + o * b[..., None]
            M = M_new
        for r in reqs:
            r.wait()
        if hop < world - 1:
            cur_k, cur_v, src = rk, rv, src_next
    return (O / L.clamp_min(1e-30)[..., None]).transpose(0, 1).to(q.dtype)


def split_sequence(n_tokens: int, world: int) -> list[tuple[int, int]]:
    """Contiguous [start, end) chunks, the first ``n % world`` one token longer."""
    base, extra = divmod(n_tokens, world)
    out, s = [], 0
    for r in range(world):
        n = base + (1 if r < extra else 0)
        out.append((s, s + n))
        s += n
    return out
