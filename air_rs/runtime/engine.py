"""Inference engine: continuous batching over the paged KV pool.

The reference serves one request at a time with batch 1 (``src/scheduler.rs:36-100``,
``src/inference_step.rs:19-184``) and keeps its Orca/Sarathi scheduler as unused
bookkeeping (``src/continuous_batch.rs``). Here the scheduler drives real batched steps:
waiting requests are admitted while KV blocks and batch slots allow, prompts are
prefilled in token-budgeted chunks (``prefill_chunk``, 2048 tokens by default: a prompt up to
that length is one GEMM pass over the weights; the reference's ``PREFILL_CHUNK_SIZE`` is 512),
and every step decodes all running sequences in one CUDA-graph
replay of the bucket that fits them. Output processing is pipelined: step k+1 is
launched before step k's tokens are read back, so the host never idles the GPU.

On a machine without CUDA the engine runs the reference-numerics CPU oracle (batch 1),
which is the reference's Candle-CPU path.
"""
from __future__ import annotations

import dataclasses
import itertools
import time
from collections import deque
from dataclasses import dataclass, field
from typing import Callable, Iterable

import numpy as np
import torch

from ..models.config import ModelConfig
from ..metrics import InferenceMetrics
from ..utils import trace


@dataclass
class SamplingParams:
    max_tokens: int = 512
    temperature: float = 0.7
    top_p: float = 0.9
    top_k: int = 40
    repetition_penalty: float = 1.1
    stop_token_ids: tuple[int, ...] = ()
    ignore_eos: bool = False


class FinishReason:
    STOP = "stop"
    LENGTH = "length"
    ERROR = "error"
    ABORT = "abort"


@dataclass
class Request:
    rid: int
    prompt_ids: list[int]
    params: SamplingParams
    priority: int = 0
    seq: int = -1                 # SequenceManager id
    slot: int = -1                # penalty-count row
    output_ids: list[int] = field(default_factory=list)
    prefilled: int = 0            # prompt tokens already in the KV cache
    finished: str | None = None
    arrival: float = field(default_factory=time.perf_counter)
    first_token_time: float | None = None
    finish_time: float | None = None
    on_token: Callable | None = None
    grammar: object | None = None
    cached_tokens: int = 0        # prompt tokens served from the prefix cache
    image_embeds: object | None = None   # [N, H] rows that replace the image placeholders
    image_token_id: int = -1

    @property
    def num_tokens(self) -> int:
        return len(self.prompt_ids) + len(self.output_ids)


BUCKETS = (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 192, 256)


class Engine:
    """Batched generation over a ``ModelRunner`` (GPU) or the CPU oracle."""

    def __init__(self, cfg: ModelConfig, runner=None, tokenizer=None, *, oracle=None,
                 max_batch: int = 64, prefill_chunk: int = 2048, max_prefill_tokens: int = 8192,
                 add_bos: bool = True, eos_id: int | None = None, prefix_cache: bool = False,
                 prefix_cache_blocks: int | None = None, kv_swap: bool = True,
                 cuda_graph_batch_sizes: tuple[int, ...] = BUCKETS, pressure_control: bool = False,
                 secure_kv: bool = False, admission: str = "fifo", arb_ratio: float = 2.0,
                 max_wait_s: float = 2.0):
        """``pressure_control``: evaluate KV-pool pressure every step and act on it (prefix-cache
        eviction from Orange, no admissions from Red, preemption at Critical)."""
        self.cfg = cfg
        self.admit_paused = False
        self.decode_ms_last = self.decode_ms_ema = None
        self.secure_kv = secure_kv        # zero the KV blocks a finished request frees
        if admission not in ("fifo", "priority", "arb"):
            raise ValueError(f"unknown admission policy {admission!r}")
        self.admission, self.arb_ratio, self.max_wait_s = admission, arb_ratio, max_wait_s
        self.buckets = tuple(sorted(cuda_graph_batch_sizes))
        self.runner = runner
        self.oracle = oracle
        self.tokenizer = tokenizer
        self.max_batch = max_batch if runner is not None else 1
        self.prefill_chunk = prefill_chunk
        self.max_prefill_tokens = max_prefill_tokens
        self.add_bos = add_bos
        self.eos_id = eos_id if eos_id is not None else cfg.eos_token_id
        self.waiting: deque[Request] = deque()
        self.running: list[Request] = []
        self.finished: dict[int, Request] = {}
        self._rid = itertools.count()
        self.metrics = InferenceMetrics()
        self.seqs = None
        self.free_slots: list[int] = []
        self.step_count = 0
        self.h2d_bytes_last_step = 0
        self.d2h_bytes_last_step = 0
        if runner is not None:
            from .. import _host  # native bookkeeping
            self.seqs = _host.SequenceManager(runner.num_blocks, runner.block_size)
            # the last penalty-count row is the sink for padding rows of a bucket
            self.pad_slot = runner.counts.shape[0] - 1
            self.free_slots = list(range(runner.counts.shape[0] - 1))[::-1]
            self._pinned: dict[int, dict] = {}
            from ..kv.prefix_cache import RadixCache
            from ..kv.swap import KvSwapManager
            self.prefix_cache = (RadixCache(runner.block_size, prefix_cache_blocks or runner.num_blocks // 2,
                                            self.seqs.allocator) if prefix_cache else None)
            self.swap = KvSwapManager(runner.kv, self.seqs) if kv_swap else None
        self.swapped: list[Request] = []      # preempted (KV in host memory), resumed first
        if runner is None:
            self.prefix_cache = self.swap = None
        self.pressure = None
        if pressure_control and runner is not None:
            from .pressure import KvPressureController
            self.pressure = KvPressureController(self)

    # ------------------------------------------------------------------ requests
    def add_request(self, prompt_ids: list[int], params: SamplingParams | None = None, *,
                    priority: int = 0, on_token: Callable | None = None, grammar=None,
                    image_embeds: torch.Tensor | None = None, image_token_id: int = -1) -> int:
        """``image_embeds`` [N, H] (e.g. ``VisionEncoder.encode`` output in the language model's
        hidden size) replace, in order, the N prompt tokens equal to ``image_token_id``."""
        params = params or SamplingParams()
        ids = list(prompt_ids)
        if self.add_bos and self.cfg.bos_token_id is not None:
            ids = [self.cfg.bos_token_id] + ids
        if self.runner is not None and len(ids) + params.max_tokens > self.runner.max_model_len:
            raise ValueError(f"prompt ({len(ids)}) + max_tokens ({params.max_tokens}) exceeds "
                             f"max_model_len {self.runner.max_model_len}")
        if image_embeds is not None:
            if self.runner is None:
                raise ValueError("image inputs need a device engine")
            n_ph = sum(1 for t in ids if t == image_token_id)
            if n_ph != image_embeds.shape[0] or image_embeds.shape[-1] != self.runner.H:
                raise ValueError(f"{n_ph} image placeholders for image embeddings of shape "
                                 f"{tuple(image_embeds.shape)} (hidden {self.runner.H})")
            image_embeds = image_embeds.to(self.runner.device, torch.float32)
        r = Request(next(self._rid), ids, params, priority=priority, on_token=on_token, grammar=grammar,
                    image_embeds=image_embeds, image_token_id=image_token_id)
        self.waiting.append(r)
        return r.rid

    def abort(self, rid: int) -> bool:
        for q in (self.waiting, self.running, self.swapped):
            for r in list(q):
                if r.rid == rid:
                    if r in self.swapped:
                        self.swapped.remove(r)
                        self.swap.drop(r.seq)
                    self._finish(r, FinishReason.ABORT)
                    if r in self.waiting:
                        self.waiting.remove(r)
                    return True
        return False

    def has_unfinished(self) -> bool:
        return bool(self.waiting or self.running or self.swapped)

    # ------------------------------------------------------------------ bookkeeping
    def _finish(self, r: Request, reason: str):
        if r.finished:
            return
        r.finished = reason
        r.finish_time = time.perf_counter()
        if r in self.running:
            self.running.remove(r)
        if getattr(self, "_defer_free", False):
            if not hasattr(self, "_deferred"):
                self._deferred = []
            self._deferred.append((r.seq, r.slot))
        else:
            if self.seqs is not None and r.seq >= 0:
                self._free_seq(r.seq)
            if r.slot >= 0:
                self.free_slots.append(r.slot)
        r.seq = -1
        r.slot = -1
        self.finished[r.rid] = r

    def _emit(self, r: Request, tok: int, prob: float = 1.0):
        if r.finished:
            return
        now = time.perf_counter()
        if r.first_token_time is None:
            r.first_token_time = now
            self.metrics.mark_first_token()
        r.output_ids.append(tok)
        self.metrics.record_token()
        if r.grammar is not None:
            try:
                r.grammar.push_token(tok)
            except Exception:
                pass
        if r.on_token is not None:
            r.on_token(r, tok)
        stop = (not r.params.ignore_eos and (tok == self.eos_id or tok in r.params.stop_token_ids))
        if r.grammar is not None and getattr(r.grammar, "is_complete", lambda: False)():
            stop = True
        if stop:
            self._finish(r, FinishReason.STOP)
        elif len(r.output_ids) >= r.params.max_tokens:
            self._finish(r, FinishReason.LENGTH)

    # ------------------------------------------------------------------ GPU scheduling
    def _admit(self) -> list[Request]:
        """Admit waiting requests while batch slots / KV blocks / token budget allow."""
        admitted = []
        if self.pressure is not None:
            self.pressure.tick()
        if self.admit_paused:
            return admitted
        budget = self.max_prefill_tokens
        alloc = self.seqs.allocator
        bs = self.runner.block_size
        reserve = sum(1 for _ in self.running)  # one growth block per running sequence
        committed = 0
        self._resume_swapped()
        if self.swapped:          # preempted requests go first
            return admitted
        while self.waiting and len(self.running) + len(admitted) < self.max_batch:
            r = self._next_waiting(admitted)
            hit, blocks = 0, []
            if self.prefix_cache is not None and r.image_embeds is None:
                # keep at least one prompt token to prefill (its logits give the first token)
                hit, blocks = self.prefix_cache.longest_prefix_match(r.prompt_ids, len(r.prompt_ids) - 1)
            need = (len(r.prompt_ids) - hit + bs - 1) // bs + 1
            if not alloc.can_allocate(need + reserve + committed) and self.prefix_cache is not None:
                self.prefix_cache.evict_until(need + reserve + committed - alloc.num_free_blocks())
            if not alloc.can_allocate(need + reserve + committed) or not self.free_slots:
                break
            if len(r.prompt_ids) - hit > budget and admitted:
                break
            self.waiting.remove(r)
            if hit:
                r.seq = self.seqs.create_with_prefix(blocks, hit)
                r.prefilled = hit
                r.cached_tokens = hit
            else:
                r.seq = self.seqs.create_sequence()
            r.slot = self.free_slots.pop()
            admitted.append(r)
            committed += need       # allocated by _prefill, after this loop
            budget -= len(r.prompt_ids) - hit
        return admitted

    def _request_for_handoff(self, prompt_ids: list[int], params: SamplingParams | None,
                             generated: list[int]) -> Request:
        """Disaggregated decode: a running request whose prompt KV arrives from a prefill
        engine (``prompt_ids`` already include BOS). Reserves the KV blocks the sender fills."""
        params = params or SamplingParams()
        if not self.free_slots:
            raise RuntimeError("no free sequence slot for a handed-over request")
        r = Request(next(self._rid), list(prompt_ids), params)
        r.seq = self.seqs.create_sequence()
        self.seqs.append(r.seq, len(prompt_ids))
        r.slot = self.free_slots.pop()
        r.prefilled = len(prompt_ids)
        self.runner.reset_counts(r.slot, torch.tensor(list(prompt_ids) + list(generated), dtype=torch.int32))
        for t in generated:
            self._emit(r, t)
        if not r.finished:
            self.running.append(r)
        return r

    # ------------------------------------------------------------------ preemption (KV host tier)
    def _blocks_needed(self, batch) -> int:
        """New KV blocks the next decode step opens (a sequence whose KV fills whole blocks)."""
        bs = self.runner.block_size
        return sum(1 for r in batch if self.seqs.num_tokens(r.seq) % bs == 0)

    def _make_room(self, batch: list) -> list:
        """Preempt the most recently admitted sequences (KV -> pinned host memory) until the
        next step's new blocks fit; returns the batch that can run."""
        alloc = self.seqs.allocator
        need = self._blocks_needed(batch)
        if need > alloc.num_free_blocks() and self.prefix_cache is not None:
            self.prefix_cache.evict_until(need - alloc.num_free_blocks())
        while batch and self._blocks_needed(batch) > alloc.num_free_blocks():
            if self.swap is None or len(batch) == 1:
                raise RuntimeError("out of KV blocks and no sequence left to preempt")
            victim = batch[-1]
            self.swap.evict(victim.seq)
            self.running.remove(victim)
            self.swapped.append(victim)
            batch = batch[:-1]
            self.metrics.preemptions = getattr(self.metrics, "preemptions", 0) + 1
        return batch

    def _next_waiting(self, admitted: list) -> "Request":
        """The waiting request the admission policy takes next.

        fifo: oldest first. priority: highest ``priority``, then oldest. arb: harmonic length
        grouping (reference ``src/batching/arb.rs``): prefer the oldest request whose prompt
        length is within ``arb_ratio`` of the running batch's median context, so one decode
        batch keeps similar attention lengths; a request older than ``max_wait_s`` goes first
        whatever its length (no starvation)."""
        if self.admission == "fifo" or len(self.waiting) == 1:
            return self.waiting[0]
        if self.admission == "priority":
            return max(self.waiting, key=lambda r: (r.priority, -r.arrival))
        now = time.perf_counter()
        oldest = self.waiting[0]
        if now - oldest.arrival > self.max_wait_s:
            return oldest
        lens = sorted(r.num_tokens for r in list(self.running) + list(admitted))
        if not lens:
            return oldest
        med = lens[len(lens) // 2]
        for r in self.waiting:
            n = len(r.prompt_ids)
            if max(n, med) <= self.arb_ratio * max(1, min(n, med)):
                return r
        return oldest

    def _timing_event(self, i: int):
        ev = getattr(self, "_tev", None)
        if ev is None:
            ev = self._tev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        return ev[i]

    def stats(self) -> dict:
        """Gauges for monitoring: queue sizes, KV pool use, prefix cache, preemptions, pressure,
        device time of the last / average decode step, collective bytes per step."""
        out = {"running": len(self.running), "waiting": len(self.waiting), "swapped": len(self.swapped),
               "decode_steps": self.step_count, "preemptions": getattr(self.metrics, "preemptions", 0)}
        from ..parallel.tp import COMM
        calls, nbytes = COMM.totals()
        out.update(collective_calls_total=calls, collective_bytes_total=nbytes)
        if self.runner is None:
            return out
        alloc = self.seqs.allocator
        total = alloc.total_blocks
        out.update(kv_blocks_total=total, kv_blocks_used=alloc.num_used_blocks(),
                   kv_utilization=alloc.num_used_blocks() / max(1, total))
        if self.prefix_cache is not None:
            st = self.prefix_cache.stats()
            out.update(prefix_cache_hit_rate=st.hit_rate, prefix_cache_blocks=st.cached_blocks,
                       prefix_cache_hit_tokens=st.hit_tokens)
        if self.pressure is not None:
            out["kv_pressure_level"] = int(self.pressure.level)
        if self.decode_ms_ema is not None:
            out.update(decode_step_device_ms=self.decode_ms_last, decode_step_device_ms_avg=self.decode_ms_ema)
        rn = self.runner
        if rn.tp_size > 1:
            # row-parallel partials cross the links twice per layer (attention output, FFN down)
            out["tp_collective_bytes_per_row"] = 2 * len(rn.w.layers) * rn.H * 4 * (rn.tp_size - 1)
        return out

    def preempt_latest(self) -> bool:
        """Swap the most recently admitted running request out to host memory."""
        if self.swap is None or not self.running:
            return False
        victim = self.running[-1]
        if victim.seq < 0 or self.seqs.is_swapped(victim.seq):
            return False
        self.swap.evict(victim.seq)
        self.running.remove(victim)
        self.swapped.append(victim)
        self.metrics.preemptions = getattr(self.metrics, "preemptions", 0) + 1
        return True

    def _resume_swapped(self):
        """Bring preempted sequences back (oldest first) while their blocks + one fit."""
        if self.admit_paused:
            return
        alloc = self.seqs.allocator
        bs = self.runner.block_size
        while self.swapped and len(self.running) < self.max_batch:
            r = self.swapped[0]
            n = (self.seqs.num_tokens(r.seq) + bs - 1) // bs
            reserve = len(self.running) + 2
            if not alloc.can_allocate(n + reserve):
                break
            self.swapped.pop(0)
            self.swap.restore(r.seq)
            self.running.append(r)

    def _prefill(self, reqs: list[Request]):
        """Chunked prefill of admitted requests; samples their first tokens."""
        rn = self.runner
        dev = rn.device
        pending = list(reqs)
        for r in pending:
            rn.reset_counts(r.slot, torch.tensor(r.prompt_ids, dtype=torch.int32))
        while pending:
            ids, pos, slots, rows, lasts, done = [], [], [], [], [], []
            seq_list, img_rows = [], []
            budget = self.max_prefill_tokens
            for i, r in enumerate(pending):
                if budget <= 0:
                    break
                n_left = len(r.prompt_ids) - r.prefilled
                n = min(n_left, self.prefill_chunk, budget)
                if n <= 0:
                    continue
                start = r.prefilled
                if r.image_embeds is not None:
                    ph = [p for p in range(start, start + n) if r.prompt_ids[p] == r.image_token_id]
                    first = sum(1 for p in range(start) if r.prompt_ids[p] == r.image_token_id)
                    img_rows.extend((len(ids) + p - start, r, first + k) for k, p in enumerate(ph))
                sl = self.seqs.append(r.seq, n)
                seq_list.append(r.seq)
                ids.extend(r.prompt_ids[start:start + n])
                pos.extend(range(start, start + n))
                slots.extend(sl)
                rows.extend([len(seq_list) - 1] * n)
                r.prefilled += n
                budget -= n
                lasts.append(len(ids) - 1)
                done.append(r if r.prefilled == len(r.prompt_ids) else None)
            tab = torch.full((len(seq_list), rn.max_blocks), -1, dtype=torch.int32)
            self.seqs.fill_table(seq_list, tab)
            S = len(lasts)
            pr = [r for r in pending if r.seq in seq_list]
            sp = [pending[i].params for i in range(len(pending)) if pending[i].seq in seq_list]
            ids_t = torch.tensor(ids, dtype=torch.int32, device=dev)
            hidden_in = None
            if img_rows:      # token embeddings with image placeholders replaced
                hidden_in = rn.embed_ids(ids_t)
                for row, r, k in img_rows:
                    hidden_in[row] = r.image_embeds[k]
            toks, probs = rn.prefill(
                ids_t,
                torch.tensor(pos, dtype=torch.int32, device=dev),
                torch.tensor(slots, dtype=torch.int64, device=dev),
                torch.tensor(rows, dtype=torch.int32, device=dev),
                tab.to(dev, non_blocking=True),
                torch.tensor(lasts, dtype=torch.int64, device=dev),
                torch.tensor([r.slot for r in pr], dtype=torch.int32, device=dev),
                torch.tensor([p.temperature for p in sp], dtype=torch.float32, device=dev),
                torch.tensor([p.repetition_penalty for p in sp], dtype=torch.float32, device=dev),
                torch.tensor([p.top_k for p in sp], dtype=torch.int32, device=dev),
                torch.tensor([p.top_p for p in sp], dtype=torch.float32, device=dev),
                mask=self._grammar_masks(pr, rn), hidden_in=hidden_in,
            )
            toks_h = toks.tolist()
            for r, d, t in zip(pr, done, toks_h):
                if d is not None:
                    if self.prefix_cache is not None and r.image_embeds is None:
                        # whole prompt blocks are complete and never written again
                        self.prefix_cache.insert(r.prompt_ids, self.seqs.block_table(r.seq))
                    self.running.append(r)
                    self._emit(r, t)
            pending = [r for r in pending if r.prefilled < len(r.prompt_ids)]
        rn.check_errors()

    def _bucket(self, n: int) -> int:
        for b in self.buckets:
            if b >= n and b <= self.runner.max_batch:
                return b
        return self.runner.max_batch

    STAGING_RING = 4

    def _pinned_for(self, B: int):
        """Per-bucket state: a ring of pinned staging slots, each guarded by an event.

        The host runs ahead of the GPU, so a staging buffer is rewritten only after the
        event recorded behind its last H2D copies has completed.
        """
        p = self._pinned.get(B)
        if p is None:
            rn = self.runner
            ring = []
            for _ in range(self.STAGING_RING):
                ring.append({
                    "i32": torch.zeros(4 * B, dtype=torch.int32).pin_memory(),
                    "slots": torch.zeros(B, dtype=torch.int64).pin_memory(),
                    "tab": torch.zeros(B, rn.max_blocks, dtype=torch.int32).pin_memory(),
                    "samp_f": torch.zeros(3 * B, dtype=torch.float32).pin_memory(),
                    "samp_i": torch.zeros(B, dtype=torch.int32).pin_memory(),
                    "tok": torch.zeros(B, dtype=torch.int32).pin_memory(),
                    "ev": None,
                })
                ring[-1]["i32_np"] = ring[-1]["i32"].numpy()        # numpy views of the pinned
                ring[-1]["slots_np"] = ring[-1]["slots"].numpy()    # buffers (vectorised fills)
            p = {"ring": ring, "next": 0, "members": None}
            self._pinned[B] = p
        return p

    def _launch_decode(self, batch: list[Request]):
        """Stage inputs (one H2D copy per buffer) and replay the bucket's graph.

        Returns (B, staging slot, event); the slot's ``tok`` receives the sampled ids once
        the event completes.
        """
        rn = self.runner
        n = len(batch)
        B = self._bucket(n)
        si = rn.step_inputs(B)
        p = self._pinned_for(B)
        st = p["ring"][p["next"]]
        p["next"] = (p["next"] + 1) % len(p["ring"])
        if st["ev"] is not None:
            st["ev"].synchronize()
        seqs = [r.seq for r in batch] + [-1] * (B - n)
        slots = self.seqs.step_slots(seqs)
        i32 = st["i32"]
        a32 = st["i32_np"]
        h2d = 0
        pos = np.fromiter((len(r.prompt_ids) + len(r.output_ids) - 1 for r in batch), dtype=np.int32, count=n)
        a32[:n] = pos
        a32[B:B + n] = pos + 1
        a32[2 * B:2 * B + n] = np.fromiter((r.slot for r in batch), dtype=np.int32, count=n)
        a32[n:B] = 0
        a32[B + n:2 * B] = 0
        a32[2 * B + n:3 * B] = self.pad_slot
        st["slots_np"][:] = slots
        si.positions.copy_(i32[:B], non_blocking=True)
        si.ctx_len.copy_(i32[B:2 * B], non_blocking=True)
        si.count_row.copy_(i32[2 * B:3 * B], non_blocking=True)
        si.slots.copy_(st["slots"], non_blocking=True)
        h2d += 3 * B * 4 + B * 8
        key = (tuple(r.rid for r in batch), tuple(r.seq for r in batch))
        if p["members"] != key:
            self.seqs.fill_table(seqs, st["tab"])
            si.block_tables.copy_(st["tab"], non_blocking=True)
            h2d += st["tab"].numel() * 4
            sf, sii = st["samp_f"], st["samp_i"]
            prs = [batch[min(i, n - 1)].params for i in range(B)]
            sf.numpy()[:] = [q.temperature for q in prs] + [q.repetition_penalty for q in prs] + [q.top_p for q in prs]
            sii.numpy()[:] = [q.top_k for q in prs]
            si.temperature.copy_(sf[:B], non_blocking=True)
            si.penalty.copy_(sf[B:2 * B], non_blocking=True)
            si.top_p.copy_(sf[2 * B:], non_blocking=True)
            si.top_k.copy_(sii, non_blocking=True)
            h2d += 4 * B * 4
            # ids: last token of each sequence (from the host; after this the graph feeds itself)
            a32[3 * B:3 * B + n] = [r.output_ids[-1] for r in batch]
            a32[3 * B + n:] = 0
            si.ids.copy_(i32[3 * B:], non_blocking=True)
            h2d += B * 4
            p["members"] = key
            p["greedy"] = all(q.temperature <= 1e-6 for q in prs)
        elif self.seqs_changed_blocks(batch):
            self.seqs.fill_table(seqs, st["tab"])
            si.block_tables.copy_(st["tab"], non_blocking=True)
            h2d += st["tab"].numel() * 4
        gm = self._grammar_masks(batch, rn, B)
        if gm is not None:
            si.mask.copy_(gm)
            self._mask_dirty = True
            h2d += gm.numel() * 4
        elif getattr(self, "_mask_dirty", False):
            for m in rn.inputs.values():
                m.mask.fill_(-1)
            self._mask_dirty = False
        rn.decode(B, use_graph=True, greedy=p.get("greedy", False))
        st["tok"].copy_(si.tokens, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        st["ev"] = ev
        self.h2d_bytes_last_step = h2d
        self.d2h_bytes_last_step = B * 4
        return B, st, ev

    def _grammar_masks(self, reqs, rn, B: int | None = None):
        """[B, ceil(V/32)] allow-bits for the sampler, or None when no request is constrained."""
        if not any(r.grammar is not None for r in reqs):
            return None
        words = (rn.V + 31) // 32
        m = torch.full((B or len(reqs), words), -1, dtype=torch.int32)
        for i, r in enumerate(reqs):
            if r.grammar is not None:
                bm = r.grammar.step_bitmask()
                m[i, : bm.numel()] = bm[:words]
        return m.to(rn.device)

    def seqs_changed_blocks(self, batch) -> bool:
        # a new block was opened for some sequence iff its new token starts a block
        bs = self.runner.block_size
        return any((r.num_tokens - 1) % bs == 0 for r in batch)

    def step(self) -> list[tuple[int, int]]:
        """One scheduler iteration; returns the (rid, token) pairs produced."""
        produced: list[tuple[int, int]] = []
        if self.runner is None:
            with trace.span("cpu_step"):
                return self._step_cpu()
        with trace.span("admit"):
            admitted = self._admit()
        if admitted:
            before = {r.rid: len(r.output_ids) for r in admitted}
            with trace.span("prefill"):
                self._prefill(admitted)
            produced += [(r.rid, r.output_ids[-1]) for r in admitted if len(r.output_ids) > before[r.rid]]
        batch = [r for r in self.running if r.output_ids and not r.finished]
        if not batch:
            return produced
        batch = self._make_room(batch)
        with trace.span("decode"):
            t0 = self._timing_event(0)
            t0.record()
            B, p, ev = self._launch_decode(batch)
            t1 = self._timing_event(1)
            t1.record()
            ev.synchronize()
            t1.synchronize()
            ms = t0.elapsed_time(t1)
            self.decode_ms_last = ms
            self.decode_ms_ema = ms if self.decode_ms_ema is None else 0.9 * self.decode_ms_ema + 0.1 * ms
        with trace.span("emit"):
            toks = p["tok"][:len(batch)].tolist()
            for r, t in zip(batch, toks):
                self._emit(r, t)
                produced.append((r.rid, t))
        self.step_count += 1
        return produced

    def run_pipelined(self, max_steps: int | None = None) -> int:
        """Decode loop that launches step k+1 before reading step k's tokens.

        The next step's inputs (positions, slots) do not depend on the sampled values (the
        graph feeds its own sampled ids forward), so output processing overlaps the GPU.
        A sequence that stops at step k still rode in step k+1; that extra token is dropped
        and its KV blocks are freed only after step k+1 has completed.
        """
        steps = 0
        inflight = None
        while max_steps is None or steps < max_steps:
            if inflight is None:
                if self.waiting:
                    admitted = self._admit()
                    if admitted:
                        self._prefill(admitted)
                if self.swapped:
                    self._resume_swapped()
                batch = [r for r in self.running if not r.finished]
                if not batch:
                    if not self.waiting and not self.swapped:
                        break
                    if self.swapped and not self.waiting:
                        self._resume_swapped()
                    continue
                batch = self._make_room(batch)
                inflight = (batch, *self._launch_decode(batch))
                continue
            ib, B, p, ev = inflight
            chain = (not self.waiting and not self.swapped and (max_steps is None or steps + 1 < max_steps) and
                     self._blocks_needed_after(ib) <= self.seqs.allocator.num_free_blocks() and
                     all(r.grammar is None for r in ib) and
                     all(len(r.output_ids) + 2 <= r.params.max_tokens for r in ib))
            nxt = None
            if chain:
                for r in ib:
                    r.output_ids.append(-1)   # the in-flight token occupies a position
                nxt = (ib, *self._launch_decode(ib))
                for r in ib:
                    r.output_ids.pop()
            ev.synchronize()
            toks = p["tok"][:len(ib)].tolist()
            for r, t in zip(ib, toks):
                self._emit_deferred(r, t)
            steps += 1
            self.step_count += 1
            if nxt is not None and any(r.finished for r in ib):
                _, _, p2, ev2 = nxt
                ev2.synchronize()
                toks = p2["tok"][:len(ib)].tolist()
                for r, t in zip(ib, toks):
                    self._emit_deferred(r, t)
                steps += 1
                self.step_count += 1
                nxt = None
            if nxt is None:
                self._release_deferred()
            inflight = nxt
        self._release_deferred()
        return steps

    def _blocks_needed_after(self, batch) -> int:
        """New blocks the step after the in-flight one opens (one more token per sequence)."""
        bs = self.runner.block_size
        return sum(1 for r in batch if self.seqs.num_tokens(r.seq) % bs == 0)

    def _emit_deferred(self, r: Request, tok: int):
        """_emit, but KV blocks of a finishing request are freed later (a step may be in flight)."""
        if r.finished:
            return
        self._defer_free = True
        try:
            self._emit(r, tok)
        finally:
            self._defer_free = False

    def _free_seq(self, seq: int):
        """Return a sequence's blocks to the pool (zeroing those it alone held with secure_kv)."""
        if self.secure_kv and not self.seqs.is_swapped(seq):
            from ..utils.security import zero_kv_blocks
            alloc = self.seqs.allocator
            zero_kv_blocks(self.runner.kv, [b for b in self.seqs.block_table(seq) if alloc.ref_count(b) == 1])
        self.seqs.free_sequence(seq)

    def _release_deferred(self):
        for seq, slot in getattr(self, "_deferred", []):
            if seq >= 0:
                self._free_seq(seq)
            if slot >= 0:
                self.free_slots.append(slot)
        self._deferred = []

    # ------------------------------------------------------------------ CPU oracle
    def _step_cpu(self):
        from ..models.reference import apply_repetition_penalty
        produced = []
        if not self.running and self.waiting:
            r = self.waiting.popleft()
            self.running.append(r)
            self.oracle.reset()
            toks = r.prompt_ids
            pc = self.prefill_chunk
            pos = 0
            if len(toks) > pc:
                n_full = len(toks) // pc * pc
                for c in range(0, n_full, pc):
                    self.oracle.forward(toks[c:c + pc], c)
                pos = n_full
                if pos == len(toks):
                    self.oracle.truncate(pos - 1)
                    pos -= 1
            r._logits = self.oracle.forward(toks[pos:], pos)
        if not self.running:
            return produced
        r = self.running[0]
        lg = apply_repetition_penalty(r._logits, r.prompt_ids + r.output_ids, r.params.repetition_penalty)
        if r.grammar is not None:
            lg = r.grammar.apply_to_logits(lg.clone())
        tok = sample_cpu(lg, r.params, self._cpu_gen())
        self._emit(r, tok)
        produced.append((r.rid, tok))
        if not r.finished:
            r._logits = self.oracle.forward([tok], r.num_tokens - 1)
        self.step_count += 1
        return produced

    def _cpu_gen(self):
        g = getattr(self, "_gen", None)
        if g is None:
            g = self._gen = torch.Generator().manual_seed(0)
        return g

    # ------------------------------------------------------------------ KV session snapshots
    def snapshot_request(self, rid: int, path) -> "object":
        """Write a running request's KV (prompt + tokens generated so far, minus the last
        sampled one, whose KV is written by the next step) to ``path``."""
        from ..kv import snapshot
        r = next((x for x in self.running if x.rid == rid), None)
        if r is None or r.seq < 0 or self.runner is None:
            raise KeyError(f"request {rid} is not running on the device")
        if self.seqs.is_swapped(r.seq):
            raise RuntimeError(f"request {rid} is swapped out")
        toks = (r.prompt_ids + r.output_ids)[: self.seqs.num_tokens(r.seq)]
        torch.cuda.current_stream(self.runner.device).synchronize()
        return snapshot.save(path, self.runner.kv, list(self.seqs.block_table(r.seq)), toks)

    def restore_snapshot(self, path) -> int:
        """Load a snapshot's whole blocks into the prefix cache; a later request whose prompt
        starts with those tokens reuses them instead of prefilling. Returns the tokens cached."""
        from ..kv import snapshot
        if self.runner is None or self.prefix_cache is None:
            raise RuntimeError("restoring a KV snapshot needs a device engine with prefix caching")
        seq, toks, blocks = snapshot.load_into(path, self.runner.kv, self.seqs)
        try:
            bs = self.runner.block_size
            n_full = len(toks) // bs
            self.prefix_cache.insert(toks[: n_full * bs], blocks[:n_full])
        finally:
            self.seqs.free_sequence(seq)
        return n_full * self.runner.block_size

    def store_prefix(self, model_id: str, rid: int, store, scheme="bf16"):
        """Keep a running request's KV (as ``snapshot_request`` selects it) in a
        ``kv.prefix_store.PrefixKvStore`` under ``model_id``."""
        r = next((x for x in self.running if x.rid == rid), None)
        if r is None or r.seq < 0 or self.runner is None:
            raise KeyError(f"request {rid} is not running on the device")
        if self.seqs.is_swapped(r.seq):
            raise RuntimeError(f"request {rid} is swapped out")
        toks = (r.prompt_ids + r.output_ids)[: self.seqs.num_tokens(r.seq)]
        torch.cuda.current_stream(self.runner.device).synchronize()
        return store.store(model_id, self.runner.kv, list(self.seqs.block_table(r.seq)), toks, scheme)

    def restore_prefix(self, model_id: str, store) -> int:
        """Load ``model_id``'s stored prefix into the prefix cache (whole blocks); returns the
        tokens cached. Lossy schemes make later outputs differ from a fresh prefill."""
        if self.runner is None or self.prefix_cache is None:
            raise RuntimeError("restoring a stored prefix needs a device engine with prefix caching")
        seq, toks, blocks = store.restore(model_id, self.runner.kv, self.seqs)
        try:
            bs = self.runner.block_size
            n_full = len(toks) // bs
            self.prefix_cache.insert(toks[: n_full * bs], blocks[:n_full])
        finally:
            self.seqs.free_sequence(seq)
        return n_full * self.runner.block_size

    # ------------------------------------------------------------------ embeddings
    def embed(self, ids: list[int]) -> list[float]:
        """Mean-pooled final-norm hidden state of a prompt (``/v1/embeddings``).

        The reference returns a hash of the input bytes here (``src/api.rs:770-780``); this is
        the model's representation.
        """
        ids = ([self.cfg.bos_token_id] if self.add_bos else []) + list(ids)
        if self.runner is None:
            return self.oracle.hidden(ids).mean(0).tolist()
        rn = self.runner
        dev = rn.device
        seq = self.seqs.create_sequence()
        try:
            slots = self.seqs.append(seq, len(ids))
            tab = torch.full((1, rn.max_blocks), -1, dtype=torch.int32)
            self.seqs.fill_table([seq], tab)
            T = len(ids)
            h = rn.prefill(torch.tensor(ids, dtype=torch.int32, device=dev),
                           torch.arange(T, dtype=torch.int32, device=dev),
                           torch.tensor(slots, dtype=torch.int64, device=dev),
                           torch.zeros(T, dtype=torch.int32, device=dev), tab.to(dev),
                           torch.tensor([T - 1], dtype=torch.int64, device=dev), None, None, None, None,
                           None, return_hidden=True)
            return h.mean(0).tolist()
        finally:
            self.seqs.free_sequence(seq)

    def token_logprobs(self, ids: list[int], add_bos: bool | None = None) -> list[float]:
        """Per-token log-probabilities of ``ids`` under the model, each given everything before
        it (BOS included when added): one forward over all rows on the GPU, teacher forcing
        on the CPU oracle. Used by the eval harness."""
        bos = self.add_bos if add_bos is None else add_bos
        ids = ([self.cfg.bos_token_id] if bos else []) + list(ids)
        T = len(ids)
        if T < 2:
            return []
        if self.runner is None:
            self.oracle.reset()
            out = []
            logits = self.oracle.forward(ids[:1], 0)
            for i in range(1, T):
                out.append(float(torch.log_softmax(logits.float(), -1)[ids[i]]))
                logits = self.oracle.forward([ids[i]], i)
            self.oracle.reset()
            return out
        rn = self.runner
        dev = rn.device
        seq = self.seqs.create_sequence()
        try:
            slots = self.seqs.append(seq, T)
            tab = torch.full((1, rn.max_blocks), -1, dtype=torch.int32)
            self.seqs.fill_table([seq], tab)
            lg = rn.prefill(torch.tensor(ids, dtype=torch.int32, device=dev),
                            torch.arange(T, dtype=torch.int32, device=dev),
                            torch.tensor(slots, dtype=torch.int64, device=dev),
                            torch.zeros(T, dtype=torch.int32, device=dev), tab.to(dev),
                            torch.arange(T - 1, dtype=torch.int64, device=dev), None, None, None, None,
                            None, return_logits=True)
            lp = torch.log_softmax(lg.float(), -1)
            tgt = torch.tensor(ids[1:], dtype=torch.long, device=dev)
            return lp.gather(1, tgt[:, None]).squeeze(1).tolist()
        finally:
            self.seqs.free_sequence(seq)

    # ------------------------------------------------------------------ high level
    def generate_ids(self, prompts: list[list[int]], params: SamplingParams | None = None,
                     pipelined: bool = False) -> list[list[int]]:
        rids = [self.add_request(p, params) for p in prompts]
        if pipelined and self.runner is not None:
            self.run_pipelined()
        while self.has_unfinished():
            self.step()
        return [self.finished[r].output_ids for r in rids]


def sample_cpu(logits: torch.Tensor, p: SamplingParams, gen: torch.Generator) -> int:
    """Host sampler with the reference's order (src/sampler.rs:83-164)."""
    if p.temperature <= 1e-6:
        return int(torch.argmax(logits))
    probs = torch.softmax(logits.float() / p.temperature, -1)
    vals, idx = torch.sort(probs, descending=True, stable=True)
    if 0 < p.top_k < vals.numel():
        vals, idx = vals[:p.top_k], idx[:p.top_k]
    if p.top_p < 1.0:
        c = torch.cumsum(vals, 0)
        cut = int(torch.searchsorted(c, torch.tensor(p.top_p)).item()) + 1
        vals, idx = vals[:cut], idx[:cut]
    total = float(vals.sum())
    if total <= 0:
        return int(torch.argmax(probs))
    r = torch.rand((), generator=gen).item() * total
    c = torch.cumsum(vals, 0)
    k = int(torch.searchsorted(c, torch.tensor(r)).item())
    return int(idx[min(k, idx.numel() - 1)])
