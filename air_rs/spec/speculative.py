"""Tree speculative decoding on the GPU runners (reference ``src/speculative.rs``).

One round for a batch of sequences:

1. **Draft tree** (EAGLE-2 constants, ``eagle2.py``): node 0 is the pending token; each
   level's frontier nodes of *all* sequences are run through the draft model in one batched
   forward whose attention rows carry ancestor bitmasks (paged tree attention), and each fed
   node gets its top-k children.
2. **Verify**: every node of every tree goes through the target in one forward with the same
   tree masks; the target's greedy next token after each node decides the longest accepted
   path, plus one bonus token.
3. **Commit / rollback**: the accepted nodes' KV entries are moved to consecutive slots and
   both sequences are truncated (block-table truncation frees the rejected branches).

Unlike the reference: tree nodes get their true RoPE positions (depth, not the shared base
position, ``src/inference_step.rs:219``), rejected draft KV is rolled back, and the draft is
not re-run once per tree node.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field

import torch

from .eagle2 import DRAFT_TOP_K, EXPAND_THRESHOLD, MAX_TREE_NODES, DraftNode, DraftTree, Eagle2Builder, greedy_accept


@dataclass
class SpecStats:
    rounds: int = 0
    drafted: int = 0
    accepted: int = 0
    emitted: int = 0
    draft_ms: float = 0.0
    verify_ms: float = 0.0

    @property
    def acceptance_rate(self) -> float:
        return self.accepted / self.drafted if self.drafted else 0.0

    @property
    def tokens_per_round(self) -> float:
        return self.emitted / self.rounds if self.rounds else 0.0

    def __str__(self):
        return (f"rounds={self.rounds} accepted/drafted={self.accepted}/{self.drafted} "
                f"({100 * self.acceptance_rate:.1f}%) tokens/round={self.tokens_per_round:.2f}")


@dataclass
class _Seq:
    tokens: list[int]                 # committed tokens; the last one is pending (not in KV)
    t_seq: int                        # target SequenceManager id
    d_seq: int                        # draft SequenceManager id
    d_len: int = 0                    # draft KV length (tokens whose KV the draft holds)
    out: list[int] = field(default_factory=list)
    done: bool = False


def copy_kv_slots(kv: torch.Tensor, block_size: int, src: list[int], dst: list[int]):
    """Move KV entries between cache slots in every layer (kv: [L, nb, 2, nkv, bs, d])."""
    pairs = [(s, d) for s, d in zip(src, dst) if s != d]
    if not pairs:
        return
    dev = kv.device
    s = torch.tensor([p[0] for p in pairs], device=dev)
    d = torch.tensor([p[1] for p in pairs], device=dev)
    vals = kv[:, s // block_size, :, :, s % block_size, :].clone()
    kv[:, d // block_size, :, :, d % block_size, :] = vals


class SpeculativeDecoder:
    def __init__(self, target, draft, k: int = 4, top_k: int = DRAFT_TOP_K, tau: float = EXPAND_THRESHOLD,
                 max_nodes: int = 32, eos_id: int | None = None, adaptive: bool = False, k_max: int = 8):
        """``target`` / ``draft``: ``air_rs.runtime.engine.Engine`` objects on the GPU.
        ``adaptive``: the draft depth follows the measured acceptance (``AcceptanceTracker``:
        longer drafts while most are accepted, shorter when they are not), within [1, k_max]."""
        if target.runner is None or (draft is not None and draft.runner is None):
            raise RuntimeError("speculative decoding needs GPU runners")
        self.t, self.d = target, draft
        self.k = k
        self.builder = Eagle2Builder(None, tau, top_k, max_depth=k + 1, max_nodes=min(max_nodes, MAX_TREE_NODES))
        self.eos_id = target.eos_id if eos_id is None else eos_id
        self.stats = SpecStats()
        self.k_max = max(k, k_max)
        self.tracker = None
        if adaptive:
            from .ghost import AcceptanceTracker
            self.tracker = AcceptanceTracker(draft_k=k)

    # -- helpers ----------------------------------------------------------------
    def _forward(self, eng, rows, seq_ids, last_rows=None):
        """rows: list of (seq index, token, position, slot, ctx_len, tree_base, tree_mask).
        Returns the logits of ``last_rows`` (all rows by default)."""
        rn = eng.runner
        dev = rn.device
        tab = torch.full((len(seq_ids), rn.max_blocks), -1, dtype=torch.int32)
        eng.seqs.fill_table(seq_ids, tab)
        T = len(rows)
        col = list(zip(*rows))
        tm = [m if m < 2**63 else m - 2**64 for m in col[6]]
        return rn.prefill(
            torch.tensor(col[1], dtype=torch.int32, device=dev),
            torch.tensor(col[2], dtype=torch.int32, device=dev),
            torch.tensor(col[3], dtype=torch.int64, device=dev),
            torch.tensor(col[0], dtype=torch.int32, device=dev), tab.to(dev),
            torch.arange(T, dtype=torch.int64, device=dev) if last_rows is None
            else torch.tensor(last_rows, dtype=torch.int64, device=dev), None, None, None, None, None,
            tree_base=torch.tensor(col[5], dtype=torch.int32, device=dev),
            tree_mask=torch.tensor(tm, dtype=torch.int64, device=dev),
            ctx_len=torch.tensor(col[4], dtype=torch.int32, device=dev), return_logits=True,
            return_final_hidden=getattr(self, "want_hidden", False) and eng is self.t)

    def _plain_prefill(self, eng, seq_id, tokens, start):
        """Feed tokens[start:] at positions start.. (no tree; all keys causal)."""
        if not tokens[start:]:
            return None
        chunk = 512
        out = None
        for c in range(start, len(tokens), chunk):
            part = tokens[c:c + chunk]
            slots = eng.seqs.append(seq_id, len(part))
            rows = [(0, tok, c + j, slots[j], c + j + 1, 1 << 30, 0) for j, tok in enumerate(part)]
            out = self._forward(eng, rows, [seq_id], last_rows=[len(rows) - 1])
        return out

    # -- public -------------------------------------------------------------------
    @torch.no_grad()
    def generate_batch(self, prompts: list[list[int]], max_tokens: int, add_bos: bool = True,
                       temperature: float = 0.0, seed: int = 0):
        """Greedy (temperature 0) or sampled generation; returns (outputs, stats).

        With temperature > 0 the target draws one token per tree node and the walk follows the
        child that matches the draw, so every emitted token is an exact sample of the target
        distribution given the accepted prefix."""
        self.temperature = temperature
        self.gen = torch.Generator(device=self.t.runner.device).manual_seed(seed)
        seqs: list[_Seq] = []
        bos = self.t.cfg.bos_token_id
        for p in prompts:
            toks = ([bos] if add_bos and bos is not None else []) + list(p)
            s = _Seq(toks, self.t.seqs.create_sequence(), self.d.seqs.create_sequence() if self.d else -1)
            # KV for all but the last (pending) token in both models
            out = self._plain_prefill(self.t, s.t_seq, toks[:-1], 0)
            self._prefilled(s, out)
            if self.d is not None:
                self._plain_prefill(self.d, s.d_seq, toks[:-1], 0)
            s.d_len = len(toks) - 1
            seqs.append(s)
        try:
            while not all(s.done for s in seqs):
                self._round([s for s in seqs if not s.done], max_tokens)
        finally:
            for s in seqs:
                self.t.seqs.free_sequence(s.t_seq)
                if self.d is not None:
                    self.d.seqs.free_sequence(s.d_seq)
        return [s.out for s in seqs], self.stats

    def generate(self, prompt: list[int], max_tokens: int, temperature: float = 0.0, add_bos: bool = True,
                 seed: int = 0):
        outs, stats = self.generate_batch([prompt], max_tokens, add_bos, temperature, seed)
        return outs[0], stats

    def _round(self, active: list[_Seq], max_tokens: int):
        t0 = time.perf_counter()
        if self.tracker is not None and self.tracker.batch_count():
            self.k = self.tracker.suggest_k(self.k_max)
            self.tracker.draft_k = self.k
            self.builder.max_depth = self.k + 1
        trees: list[DraftTree] = []
        for s in active:
            P = len(s.tokens) - 1
            # draft catch-up: tokens committed since the draft's KV ends (bonus tokens)
            if s.d_len < P:
                self.d.seqs.truncate(s.d_seq, s.d_len)
                self._plain_prefill(self.d, s.d_seq, s.tokens[:P], s.d_len)
                s.d_len = P
            tr = DraftTree(s.tokens[-1])
            tr.nodes.append(DraftNode(s.tokens[-1], 1.0, 0, None, 1.0))
            trees.append(tr)
        # ---- draft: level by level, all sequences together ----
        frontier = [[0] for _ in active]
        fed = [set() for _ in active]
        for level in range(self.k):
            rows, owners = [], []
            for si, (s, tr, fr) in enumerate(zip(active, trees, frontier)):
                P = len(s.tokens) - 1
                for node in fr:
                    need = P + node + 1 - self.d.seqs.num_tokens(s.d_seq)
                    if need > 0:
                        self.d.seqs.append(s.d_seq, need)
                    slot = self.d.seqs.slot(s.d_seq, P + node)
                    bits = tr.ancestor_bits()[node]
                    rows.append((si, tr.nodes[node].token_id, P + tr.nodes[node].depth, slot, P + node + 1, P, bits))
                    owners.append((si, node))
            if not rows:
                break
            logits = self._forward(self.d, rows, [s.d_seq for s in active])
            v, ix = torch.topk(torch.softmax(logits.float(), -1), self.builder.top_k, dim=-1)
            v, ix = v.tolist(), ix.tolist()
            nxt = [[] for _ in active]
            for (si, node), vr, ir in zip(owners, v, ix):
                fed[si].add(node)
                nxt[si].extend(self.builder.add_children(trees[si], node, list(zip(ir, vr))))
            frontier = nxt
        t1 = time.perf_counter()
        self._verify_commit(active, trees, fed, max_tokens)
        self.stats.rounds += 1
        self.stats.draft_ms += (t1 - t0) * 1e3
        self.stats.verify_ms += (time.perf_counter() - t1) * 1e3

    def _verify_commit(self, active: list[_Seq], trees: list[DraftTree], fed: list[set], max_tokens: int):
        """Target forward over every tree node, greedy / sampled acceptance, KV compaction of
        the accepted path and rollback of the rest (target and, when present, draft)."""
        # ---- verify: every node of every tree in one target forward ----
        rows, owners = [], []
        for si, (s, tr) in enumerate(zip(active, trees)):
            P = len(s.tokens) - 1
            n = len(tr.nodes)
            self.t.seqs.append(s.t_seq, P + n - self.t.seqs.num_tokens(s.t_seq))
            bits = tr.ancestor_bits()
            for i, nd in enumerate(tr.nodes):
                rows.append((si, nd.token_id, P + nd.depth, self.t.seqs.slot(s.t_seq, P + i), P + i + 1, P, bits[i]))
                owners.append((si, i))
        logits = self._forward(self.t, rows, [s.t_seq for s in active])
        if isinstance(logits, tuple):
            logits, self._verify_hidden = logits
        if self.temperature > 0:
            pr = torch.softmax(logits.float() / self.temperature, -1)
            tnext = torch.multinomial(pr, 1, generator=self.gen).squeeze(1).tolist()
        else:
            tnext = logits.argmax(-1).tolist()
        per_seq = [[0] * len(tr.nodes) for tr in trees]
        for (si, i), tok in zip(owners, tnext):
            per_seq[si][i] = tok
        self._after_verify(active, trees, logits, owners)
        # ---- accept, compact, roll back ----
        for si, (s, tr) in enumerate(zip(active, trees)):
            P = len(s.tokens) - 1
            path, bonus = greedy_accept(tr, per_seq[si])
            new_tokens = [tr.nodes[i].token_id for i in path[1:]] + [bonus]
            self.stats.drafted += len(tr.nodes) - 1
            self.stats.accepted += len(path) - 1
            if self.tracker is not None:
                depth = max((nd.depth for nd in tr.nodes), default=0)
                self.tracker.report_batch(depth, len(path) - 1)
            # target: accepted nodes -> slots P .. P+len(path)-1
            src = [self.t.seqs.slot(s.t_seq, P + i) for i in path]
            self.t.seqs.truncate(s.t_seq, P + len(path))
            dst = [self.t.seqs.slot(s.t_seq, P + j) for j in range(len(path))]
            copy_kv_slots(self.t.runner.kv, self.t.runner.block_size, src, dst)
            self._accepted(si, s, path)
            if self.d is not None:
                # draft: keep the longest prefix of the path that the draft has fed
                keep = 0
                while keep < len(path) and path[keep] in fed[si]:
                    keep += 1
                srcd = [self.d.seqs.slot(s.d_seq, P + i) for i in path[:keep]]
                self.d.seqs.truncate(s.d_seq, P + keep)
                dstd = [self.d.seqs.slot(s.d_seq, P + j) for j in range(keep)]
                copy_kv_slots(self.d.runner.kv, self.d.runner.block_size, srcd, dstd)
                s.d_len = P + keep
            for tok in new_tokens:
                if s.done:
                    break
                s.out.append(tok)
                s.tokens.append(tok)
                self.stats.emitted += 1
                if len(s.out) >= max_tokens or (self.eos_id is not None and tok == self.eos_id):
                    s.done = True

    # hooks for drafters that read the target's own hidden states (Medusa)
    def _prefilled(self, s: _Seq, out):
        pass

    def _after_verify(self, active, trees, logits, owners):
        pass

    def _accepted(self, si: int, s: _Seq, path: list[int]):
        pass
