"""Vocabulary-parallel sampling: each tensor-parallel rank holds a [B, V/W] slice of the
logits (the vocab-parallel LM head's output) and the ranks agree on the sampled tokens after
exchanging a few candidates per row instead of all-gathering [B, V] logits.

The reference gathers nothing (its ``--tp`` runs rank 0 alone, ``src/generator.rs:211-213``)
and samples on the host (``src/sampler.rs``: repetition penalty, temperature, top-k, top-p).
Here, per step:

1. each rank applies the repetition penalty and the token mask to its slice, scales by
   1/temperature, and takes its top ``C`` (value, global index) pairs and the log-sum-exp of
   its whole slice;
2. one ``all_gather`` of [B, 2C + 1] floats per rank (C = 64: 516 B per row per rank versus
   4 V bytes for the logits, 512 KB at V = 128K);
3. every rank merges the W x C candidates identically: the global top C, the global
   log-sum-exp, exact probabilities ``exp(l - lse)`` of the candidates;
4. greedy rows take the best candidate (lowest index on ties, as a full argmax); sampled rows
   keep the first ``top_k`` candidates (top_k <= C), cut the nucleus at ``top_p`` and draw with
   a uniform from a generator seeded by (seed, step), identical on every rank.

The candidates are exact for top-k rows and for nucleus rows whose nucleus fits in C tokens.
A top_k = 0 row whose nucleus is wider than the candidates, or whose whole-vocabulary draw
lands beyond their probability mass, is drawn over the full vocabulary after one
``all_gather`` of its logits; every rank holds the same candidates and uniform, so all of them
take that branch together.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

DEFAULT_CANDIDATES = 64


@dataclass
class VocabShard:
    rank: int
    world: int
    vocab: int             # real vocabulary size
    shard: int             # columns per rank (the last rank's tail may be padding)

    @property
    def start(self) -> int:
        return self.rank * self.shard

    def valid(self) -> int:
        return max(0, min(self.shard, self.vocab - self.start))


def _prepare(local: torch.Tensor, sh: VocabShard, temperature: torch.Tensor, counts=None, penalty=None,
             mask=None) -> torch.Tensor:
    """Penalised, masked, temperature-scaled float32 slice; padding columns at -inf."""
    x = local.float().clone()
    nv = sh.valid()
    if nv < x.shape[1]:
        x[:, nv:] = float("-inf")
    if counts is not None and penalty is not None:
        seen = counts[:, sh.start:sh.start + x.shape[1]].to(x.device) > 0
        if seen.shape[1] < x.shape[1]:
            seen = torch.nn.functional.pad(seen, (0, x.shape[1] - seen.shape[1]))
        p = penalty.float().to(x.device)[:, None]
        x = torch.where(seen, torch.where(x > 0, x / p, x * p), x)
    if mask is not None:
        m = mask[:, sh.start:sh.start + x.shape[1]].to(x.device)
        if m.shape[1] < x.shape[1]:
            m = torch.nn.functional.pad(m, (0, x.shape[1] - m.shape[1]))
        x = x.masked_fill(~m, float("-inf"))
    t = temperature.float().to(x.device)
    return x / torch.where(t > 0, t, torch.ones_like(t))[:, None]


def _uniform(seed: int, step: int, B: int) -> torch.Tensor:
    g = torch.Generator().manual_seed((int(seed) * 1_000_003 + int(step)) & 0x7FFF_FFFF_FFFF_FFFF)
    return torch.rand(B, generator=g, dtype=torch.float64)


def _pick(probs_sorted: torch.Tensor, u: float) -> int:
    """Index into the (descending) kept probabilities for a uniform u in [0, 1)."""
    c = torch.cumsum(probs_sorted.double(), 0)
    c = c / c[-1]
    return int(torch.searchsorted(c, torch.tensor([u], dtype=torch.float64)).clamp_max(c.numel() - 1))


def _nucleus(p: torch.Tensor, top_k: int, top_p: float) -> int:
    """Number of leading (descending) probabilities kept by top-k then top-p."""
    n = p.numel() if top_k <= 0 else min(top_k, p.numel())
    if top_p < 1.0:
        c = torch.cumsum(p[:n].double(), 0)
        n = min(n, int((c < top_p).sum()) + 1)
    return max(1, n)


def sample_full(logits: torch.Tensor, temperature, top_k, top_p, seed: int, step: int, counts=None,
                penalty=None, mask=None, vocab: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """The same rule over whole [B, V] logits (the 1-rank case): (tokens [B], probs [B])."""
    V = vocab or logits.shape[1]
    sh = VocabShard(0, 1, V, logits.shape[1])
    x = _prepare(logits, sh, temperature, counts, penalty, mask).double()
    u = _uniform(seed, step, x.shape[0])
    toks, probs = [], []
    for b in range(x.shape[0]):
        row = x[b]
        if float(temperature[b]) <= 0:
            i = int(torch.argmax(row))
            toks.append(i)
            probs.append(1.0)
            continue
        p = torch.softmax(row, 0)
        ps, ix = torch.sort(p, descending=True, stable=True)
        n = _nucleus(ps, int(top_k[b]), float(top_p[b]))
        j = _pick(ps[:n], float(u[b]))
        toks.append(int(ix[j]))
        probs.append(float(ps[j]))
    return torch.tensor(toks, dtype=torch.int64), torch.tensor(probs, dtype=torch.float32)


class VocabParallelSampler:
    """Agrees on sampled tokens across the ranks of ``group`` from their logit slices."""

    def __init__(self, vocab: int, shard: int, group=None, candidates: int = DEFAULT_CANDIDATES):
        self.group = group
        self.sh = VocabShard(dist.get_rank(group), dist.get_world_size(group), vocab, shard)
        self.C = min(candidates, shard)
        self.fallbacks = 0
        self.bytes_exchanged = 0

    def sample(self, local: torch.Tensor, temperature, top_k, top_p, seed: int, step: int, counts=None,
               penalty=None, mask=None) -> tuple[torch.Tensor, torch.Tensor]:
        sh, C = self.sh, self.C
        if int(torch.as_tensor(top_k).max()) > C:
            raise ValueError(f"top_k above the {C} candidates per rank")
        x = _prepare(local, sh, temperature, counts, penalty, mask)
        B = x.shape[0]
        v, i = torch.topk(x, C, dim=1)                       # descending, per rank
        lse = torch.logsumexp(x.double(), 1).float()
        pack = torch.cat([v, (i + sh.start).float(), lse[:, None]], 1).contiguous()   # [B, 2C + 1]
        allp = [torch.empty_like(pack) for _ in range(sh.world)]
        dist.all_gather(allp, pack, group=self.group)
        self.bytes_exchanged += pack.numel() * 4 * sh.world
        cv = torch.cat([a[:, :C] for a in allp], 1).double()               # [B, W C]
        ci = torch.cat([a[:, C:2 * C] for a in allp], 1).round().long()
        glse = torch.logsumexp(torch.stack([a[:, 2 * C] for a in allp], 1).double(), 1)
        # global order: value descending, index ascending on ties (a full argmax's choice)
        key = torch.argsort(ci, dim=1, stable=True)
        cv, ci = cv.gather(1, key), ci.gather(1, key)
        order = torch.argsort(-cv, dim=1, stable=True)[:, :C]
        cv, ci = cv.gather(1, order), ci.gather(1, order)
        u = _uniform(seed, step, B)
        toks = torch.empty(B, dtype=torch.int64)
        probs = torch.empty(B, dtype=torch.float32)
        for b in range(B):
            if float(temperature[b]) <= 0:
                toks[b], probs[b] = int(ci[b, 0]), 1.0
                continue
            p = torch.exp(cv[b] - glse[b])                                # exact probabilities
            k, tp, ub = int(top_k[b]), float(top_p[b]), float(u[b])
            mass = float(p.sum())
            if k <= 0 and tp >= 1.0:
                # whole-vocabulary draw: the candidates hold the first `mass` of it exactly
                if ub >= mass:
                    toks[b], probs[b] = self._full_row(x[b], tp, ub)
                    continue
                j = int(torch.searchsorted(torch.cumsum(p, 0), torch.tensor([ub], dtype=torch.float64)))
            elif k <= 0 and mass < tp:
                toks[b], probs[b] = self._full_row(x[b], tp, ub)       # nucleus wider than C
                continue
            else:
                j = _pick(p[:_nucleus(p, k, tp)], ub)
            toks[b], probs[b] = int(ci[b, j]), float(p[j])
        return toks, probs

    def _full_row(self, row: torch.Tensor, top_p: float, u: float) -> tuple[int, float]:
        """Gather one row's whole logits and draw over the full vocabulary (every rank does
        the same, in the same order)."""
        self.fallbacks += 1
        parts = [torch.empty_like(row) for _ in range(self.sh.world)]
        dist.all_gather(parts, row.contiguous(), group=self.group)
        self.bytes_exchanged += row.numel() * 4 * self.sh.world
        full = torch.cat(parts)[: self.sh.vocab].double()
        p = torch.softmax(full, 0)
        ps, ix = torch.sort(p, descending=True, stable=True)
        n = _nucleus(ps, 0, top_p)
        j = _pick(ps[:n], u)
        return int(ix[j]), float(ps[j])
