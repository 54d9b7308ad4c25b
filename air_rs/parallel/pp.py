"""Pipeline parallelism for inference (reference ``src/pipeline_parallel.rs`` PipelineRunner
threads over in-process channels, ``src/gpu_pipeline.rs`` even layer partitioning).

One process per stage (one GPU or one TP group per stage). Each stage's runner holds a
contiguous layer range (``build_runner(layer_range=...)``) and its slice of the KV pool.
Micro-batches flow forward over ``torch.distributed`` point-to-point sends (NCCL on GPUs,
gloo on CPU): stage i receives the residual stream of micro-batch m from stage i-1, runs
its layers, and posts a non-blocking send to stage i+1 before taking micro-batch m+1, so
stage i works on m+1 while stage i+1 works on m. The last stage samples; its tokens are
broadcast to every stage so the (identical, deterministic) host bookkeeping of all stages
stays in step.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.distributed as dist


def partition_layers(n_layers: int, n_stages: int) -> list[tuple[int, int]]:
    """Even split; the first ``n_layers % n_stages`` stages take one extra layer."""
    base, extra = divmod(n_layers, n_stages)
    out, s = [], 0
    for i in range(n_stages):
        n = base + (1 if i < extra else 0)
        out.append((s, s + n))
        s += n
    return out


@dataclass
class MicroBatch:
    ids: torch.Tensor             # [T] int32
    positions: torch.Tensor       # [T] int32
    slots: torch.Tensor           # [T] int64
    row_seq: torch.Tensor         # [T] int32
    block_tables: torch.Tensor    # [S, max_blocks] int32
    last_rows: torch.Tensor       # [S] int64
    count_rows: torch.Tensor      # [S] int32
    extra: dict = field(default_factory=dict)

    @property
    def T(self) -> int:
        return self.ids.numel()

    @property
    def S(self) -> int:
        return self.last_rows.numel()


class PipelineRunner:
    """Moves micro-batches through ``stage.forward(mb, hidden_in) -> hidden | tokens``."""

    def __init__(self, stage, rank: int, world: int, hidden: int, device, group=None):
        self.stage, self.rank, self.world, self.hidden = stage, rank, world, hidden
        self.device = torch.device(device)
        self.group = group
        self.first, self.last = rank == 0, rank == world - 1
        self.sent_bytes = 0

    def _peer(self, r):
        return dist.get_global_rank(self.group, r) if self.group is not None else r

    def run(self, mbs: list[MicroBatch]) -> list[torch.Tensor]:
        pending, outs = [], []
        for mb in mbs:
            h = None
            if not self.first:
                h = torch.empty(mb.T, self.hidden, dtype=torch.float32, device=self.device)
                dist.recv(h, src=self._peer(self.rank - 1), group=self.group)
            y = self.stage.forward(mb, h)
            if self.last:
                outs.append(y.to(torch.int32))
            else:
                pending.append((dist.isend(y.contiguous(), dst=self._peer(self.rank + 1), group=self.group), y))
                self.sent_bytes += y.numel() * y.element_size()
        for work, _ in pending:
            work.wait()
        res = []
        for i, mb in enumerate(mbs):
            t = outs[i] if self.last else torch.empty(mb.S, dtype=torch.int32, device=self.device)
            if self.world > 1:
                dist.broadcast(t, src=self._peer(self.world - 1), group=self.group)
            res.append(t)
        return res


class RunnerStage:
    """A ``ModelRunner`` holding one stage's layers (greedy / sampled via its device sampler)."""

    def __init__(self, runner, first: bool, last: bool):
        self.rn, self.first, self.last = runner, first, last

    def forward(self, mb: MicroBatch, hidden_in):
        rn, dev = self.rn, self.rn.device
        S = mb.S
        out = rn.prefill(mb.ids, mb.positions, mb.slots, mb.row_seq, mb.block_tables, mb.last_rows,
                         mb.count_rows, mb.extra.get("temperature", torch.zeros(S, device=dev)),
                         mb.extra.get("penalty", torch.ones(S, device=dev)),
                         mb.extra.get("top_k", torch.zeros(S, dtype=torch.int32, device=dev)),
                         mb.extra.get("top_p", torch.ones(S, device=dev)),
                         hidden_in=hidden_in, return_hidden_out=not self.last)
        return out if not self.last else out[0]


class PipelineEngine:
    """Batched greedy/sampled generation over a pipeline; every stage calls ``generate`` with
    the same prompts (deterministic bookkeeping, tokens broadcast from the last stage)."""

    def __init__(self, runner, rank: int, world: int, micro_batches: int = 2, group=None, bos: int | None = None):
        from .. import _host
        self.rn = runner
        self.seqs = _host.SequenceManager(runner.num_blocks, runner.block_size)
        self.pipe = PipelineRunner(RunnerStage(runner, rank == 0, rank == world - 1), rank, world,
                                   runner.H, runner.device, group)
        self.M = micro_batches
        self.bos = bos

    def _mb(self, rows: list[tuple[int, list[int], int]], seq_ids: list[int], count_rows: list[int],
            temperature: float, penalty: float) -> MicroBatch:
        """rows: (seq index within mb, token ids, start position)."""
        rn, dev = self.rn, self.rn.device
        ids, pos, slots, rseq, lasts = [], [], [], [], []
        for si, toks, start in rows:
            sl = self.seqs.append(seq_ids[si], len(toks))
            ids += toks
            pos += list(range(start, start + len(toks)))
            slots += sl
            rseq += [si] * len(toks)
            lasts.append(len(ids) - 1)
        tab = torch.full((len(seq_ids), rn.max_blocks), -1, dtype=torch.int32)
        self.seqs.fill_table(seq_ids, tab)
        S = len(seq_ids)
        f = lambda v: torch.full((S,), v, dtype=torch.float32, device=dev)
        return MicroBatch(torch.tensor(ids, dtype=torch.int32, device=dev),
                          torch.tensor(pos, dtype=torch.int32, device=dev),
                          torch.tensor(slots, dtype=torch.int64, device=dev),
                          torch.tensor(rseq, dtype=torch.int32, device=dev), tab.to(dev),
                          torch.tensor(lasts, dtype=torch.int64, device=dev),
                          torch.tensor(count_rows, dtype=torch.int32, device=dev),
                          {"temperature": f(temperature), "penalty": f(penalty)})

    def generate(self, prompts: list[list[int]], max_tokens: int, temperature: float = 0.0,
                 penalty: float = 1.0) -> list[list[int]]:
        rn = self.rn
        prompts = [([self.bos] if self.bos is not None else []) + list(p) for p in prompts]
        n = len(prompts)
        groups = [list(range(g, n, self.M)) for g in range(min(self.M, n))]
        seq_ids = [self.seqs.create_sequence() for _ in range(n)]
        if self.pipe.last:
            for i, p in enumerate(prompts):
                rn.reset_counts(i, torch.tensor(p, dtype=torch.int32))
        outs: list[list[int]] = [[] for _ in range(n)]
        try:
            mbs = [self._mb([(j, prompts[i], 0) for j, i in enumerate(g)], [seq_ids[i] for i in g], g,
                            temperature, penalty) for g in groups]
            for g, t in zip(groups, self.pipe.run(mbs)):
                for i, tok in zip(g, t.tolist()):
                    outs[i].append(tok)
            for _ in range(max_tokens - 1):
                mbs = [self._mb([(j, [outs[i][-1]], len(prompts[i]) + len(outs[i]) - 1) for j, i in enumerate(g)],
                                [seq_ids[i] for i in g], g, temperature, penalty) for g in groups]
                for g, t in zip(groups, self.pipe.run(mbs)):
                    for i, tok in zip(g, t.tolist()):
                        outs[i].append(tok)
        finally:
            for s in seq_ids:
                self.seqs.free_sequence(s)
        return outs
