"""Medusa heads and the CDSC speculative council (reference ``src/medusa_heads.rs``,
``src/speculative_council.rs``, ``src/async_verifier.rs``).

Both drafters reuse ``SpeculativeDecoder``'s tree verification on the target model (one
forward over every draft node with ancestor masks, greedy or exact sampled acceptance, KV
compaction and rollback), so the acceptance statistics are the target's real decisions —
the reference's council verifier accepted by a hash of the token ids.

* ``MedusaDecoder``: K extra heads on the target's own final hidden state. Head k maps the
  hidden h_t of the last accepted position to logits for token t+1+k through a residual
  SwiGLU block and the target's LM head (``lm(h + silu(h W1^T) * (h W2^T))``); the draft tree takes the
  top-c tokens of each head as the children of every node of the previous depth (cumulative
  probability order, capped node count). Heads are random-initialised here (no trained
  checkpoints offline) and load from the reference's GGUF tensors ``mtp_head.{i}.weight0/1``
  or from a ``.pt`` state dict with a ``.draft.json`` manifest.
* ``CouncilDecoder`` (``--council``, ``--epsilon``): several voter drafts (draft engines)
  propose the next token; the council extends a draft chain only while the voters agree —
  the Jensen-Shannon divergence of their distributions is at most epsilon — with the
  argmax of the mean distribution, and stops drafting at the first disagreement.
"""
from __future__ import annotations

import math
import time

import torch

from .eagle2 import DraftNode, DraftTree
from .speculative import MAX_TREE_NODES, SpeculativeDecoder, _Seq


class MedusaHeads:
    """K draft heads, each one residual SwiGLU block on the final hidden state:
    ``h' = h + silu(h W1^T) * (h W2^T)``, then the target's LM head (reference
    ``src/medusa_heads.rs:71-94``). Weights are [hidden, hidden] pairs; random init uses
    N(0, 1/hidden) like the reference's bootstrap heads."""

    def __init__(self, hidden: int, n_heads: int = 3, device="cuda", seed: int = 0, dtype=torch.float32,
                 init_scale: float | None = None):
        g = torch.Generator().manual_seed(seed)
        sc = init_scale if init_scale is not None else 1.0 / math.sqrt(hidden)
        mk = lambda: (torch.randn(hidden, hidden, generator=g) * sc).to(device, dtype)
        self.W = [(mk(), mk()) for _ in range(n_heads)]
        self.n_heads = n_heads

    @staticmethod
    def _from_pairs(ws, device) -> "MedusaHeads":
        obj = MedusaHeads.__new__(MedusaHeads)
        obj.W = [(a.to(device, torch.float32), b.to(device, torch.float32)) for a, b in ws]
        obj.n_heads = len(ws)
        return obj

    @classmethod
    def from_gguf(cls, path: str, n_heads: int | None = None, device="cuda") -> "MedusaHeads":
        """Native multi-token heads stored in a GGUF checkpoint as ``mtp_head.{i}.weight0`` (W1)
        and ``mtp_head.{i}.weight1`` (W2), the names the reference loads
        (``src/medusa_heads.rs:137-160``). Heads are read in index order until one is missing
        (or ``n_heads`` are read); a file with none raises."""
        from ..gguf import read_gguf
        f = read_gguf(path)
        try:
            ws, i = [], 0
            while (n_heads is None or i < n_heads) and f.has(f"mtp_head.{i}.weight0"):
                if not f.has(f"mtp_head.{i}.weight1"):
                    raise ValueError(f"{path}: mtp_head.{i}.weight1 is missing")
                ws.append((f.dequantize(f"mtp_head.{i}.weight0").float(),
                           f.dequantize(f"mtp_head.{i}.weight1").float()))
                i += 1
        finally:
            f.close()
        if not ws:
            raise ValueError(f"{path}: no mtp_head.<i>.weight0/weight1 tensors")
        if n_heads is not None and len(ws) < n_heads:
            raise ValueError(f"{path}: {n_heads} heads requested, {len(ws)} present")
        hid = ws[0][0].shape[0]
        if any(tuple(t.shape) != (hid, hid) for pair in ws for t in pair):
            raise ValueError(f"{path}: MTP heads are not square and equal-sized")
        return cls._from_pairs(ws, device)

    @classmethod
    def load(cls, path: str, device="cuda", fingerprint: bytes | None = None,
             hidden: int | None = None) -> "MedusaHeads":
        """Heads from a ``.gguf`` (``from_gguf``) or a torch state dict (keys ``head<i>.w1`` /
        ``head<i>.w2``). A ``<path>.draft.json`` manifest next to a state dict, when present,
        must match ``fingerprint`` (the target checkpoint's, ``parallel.pd.gguf_fingerprint``)
        and ``hidden``, and the heads must match the manifest."""
        import json
        import os
        import re
        if path.endswith(".gguf"):
            heads = cls.from_gguf(path, device=device)
            if hidden is not None and heads.W[0][0].shape[0] != hidden:
                raise ValueError(f"{path}: heads are not {hidden} x {hidden}")
            return heads
        sd = torch.load(path, map_location="cpu", weights_only=True)
        idx = {}
        for k in sd:
            m = re.fullmatch(r"head(\d+)\.w([12])", k)
            if m is None:
                raise ValueError(f"{path}: unexpected key {k!r} (expected head<i>.w1 / head<i>.w2)")
            idx.setdefault(int(m.group(1)), {})[m.group(2)] = sd[k]
        if not idx or sorted(idx) != list(range(len(idx))) or any(len(v) != 2 for v in idx.values()):
            raise ValueError(f"{path}: heads must be numbered 0..n-1, each with w1 and w2")
        ws = [(idx[i]["1"], idx[i]["2"]) for i in range(len(idx))]
        man_path = path + ".draft.json"
        if os.path.exists(man_path):
            with open(man_path) as f:
                man = json.load(f)
            if fingerprint is not None and man.get("target_fingerprint") not in (None, bytes(fingerprint).hex()):
                raise ValueError(f"{path}: draft heads were trained for another target ({man.get('target_name')!r})")
            if man.get("n_heads") != len(ws) or any(tuple(w.shape) != (man["hidden"], man["hidden"])
                                                    for pair in ws for w in pair):
                raise ValueError(f"{path}: heads do not match their manifest")
        if hidden is not None and any(tuple(w.shape) != (hidden, hidden) for pair in ws for w in pair):
            raise ValueError(f"{path}: heads are not {hidden} x {hidden}")
        return cls._from_pairs(ws, device)

    def state_dict(self) -> dict:
        sd = {}
        for i, (a, b) in enumerate(self.W):
            sd[f"head{i}.w1"], sd[f"head{i}.w2"] = a.cpu(), b.cpu()
        return sd

    def save(self, path: str, fingerprint: bytes | None = None, target_name: str = "") -> str:
        """State dict at ``path`` plus the ``<path>.draft.json`` manifest (kind, head count,
        hidden size, target checkpoint fingerprint and name); returns the manifest path."""
        import json
        torch.save(self.state_dict(), path)
        man = {"kind": "medusa", "n_heads": self.n_heads, "hidden": int(self.W[0][0].shape[0]),
               "target_fingerprint": None if fingerprint is None else bytes(fingerprint).hex(),
               "target_name": target_name}
        with open(path + ".draft.json", "w") as f:
            json.dump(man, f, indent=1)
        return path + ".draft.json"

    def hidden(self, h: torch.Tensor) -> list[torch.Tensor]:
        """h [S, H] -> per head the transformed hidden state [S, H]."""
        return [h + torch.nn.functional.silu(h @ w1.t()) * (h @ w2.t()) for w1, w2 in self.W]

    def logits(self, h: torch.Tensor, lm_head_fn) -> list[torch.Tensor]:
        """h [S, H] final-norm hidden -> per head [S, V] logits."""
        return [lm_head_fn(t) for t in self.hidden(h)]


class MedusaDecoder(SpeculativeDecoder):
    def __init__(self, target, heads: MedusaHeads, top_c: int = 2, max_nodes: int = 16, eos_id=None,
                 monitor=None):
        super().__init__(target, None, k=heads.n_heads, max_nodes=max_nodes, eos_id=eos_id)
        self.heads, self.top_c = heads, top_c
        # optional spec.wavefront.WavefrontHealthMonitor: acceptance per verified path sets
        # the node budget of the next draft tree
        self.monitor = monitor
        self.want_hidden = True
        self._hidden: dict[int, torch.Tensor] = {}
        rn = target.runner
        from ..ops import gemm
        self._lm = lambda x: gemm.linear(x.to(torch.bfloat16).contiguous(), rn.w.lm_head,
                                         torch.zeros(x.shape[0], rn.V_l, device=rn.device), rn)[:, : rn.V].float()

    def _prefilled(self, s: _Seq, out):
        # hidden of the position before the pending token (the prompt's second-to-last)
        self._hidden[id(s)] = out[1][-1] if isinstance(out, tuple) else None

    def _round(self, active, max_tokens):
        t0 = time.perf_counter()
        trees, fed = [], []
        for s in active:
            tr = DraftTree(s.tokens[-1], [DraftNode(s.tokens[-1], 1.0, 0, None, 1.0)])
            h = self._hidden.get(id(s))
            if h is not None:
                frontier = [0]
                for lg in self.heads.logits(h[None], self._lm):
                    p = torch.softmax(lg[0], -1)
                    v, ix = torch.topk(p, self.top_c)
                    nxt = []
                    for parent in frontier:
                        for tok, q in zip(ix.tolist(), v.tolist()):
                            if len(tr.nodes) >= self.builder.max_nodes:
                                break
                            tr.nodes.append(DraftNode(tok, q, tr.nodes[parent].depth + 1, parent,
                                                      tr.nodes[parent].cum_prob * q))
                            nxt.append(len(tr.nodes) - 1)
                    frontier = nxt
            trees.append(tr)
            fed.append(set())
        t1 = time.perf_counter()
        self._verify_commit(active, trees, fed, max_tokens)
        self.stats.rounds += 1
        self.stats.draft_ms += (t1 - t0) * 1e3
        self.stats.verify_ms += (time.perf_counter() - t1) * 1e3

    def _after_verify(self, active, trees, logits, owners):
        self._owners = owners

    def _accepted(self, si, s, path):
        if self.monitor is not None:
            self.monitor.update(len(path) - 1, self.heads.n_heads)
            self.builder.max_nodes = min(MAX_TREE_NODES, max(2, self.monitor.current_draft_size))
        # the last accepted node's hidden drives the next round's heads
        hid = getattr(self, "_verify_hidden", None)
        if hid is None:
            return
        row = [k for k, (sj, i) in enumerate(self._owners) if sj == si and i == path[-1]][0]
        self._hidden[id(s)] = hid[row]


def jsd(dists: list[torch.Tensor]) -> float:
    """Generalised Jensen-Shannon divergence (nats) of several distributions."""
    m = torch.stack(dists).mean(0)
    def kl(p):
        mask = p > 0
        return float((p[mask] * (p[mask].log() - m[mask].clamp_min(1e-30).log())).sum())
    return sum(kl(p) for p in dists) / len(dists)


class CouncilDecoder(SpeculativeDecoder):
    """Consensus drafting over ``voters`` (draft engines sharing the tokenizer)."""

    def __init__(self, target, voters: list, epsilon: float = 0.15, k: int = 4, eos_id=None):
        super().__init__(target, voters[0], k=k, max_nodes=k + 1, eos_id=eos_id)
        self.voters, self.epsilon = voters, epsilon
        self.jsd_history: list[float] = []
        self._vseq: dict[tuple[int, int], int] = {}

    def _voter_dists(self, vi: int, eng, s: _Seq, chain: list[int]) -> torch.Tensor:
        """Next-token distribution of voter vi after ``s.tokens + chain`` (its own KV)."""
        key = (id(s), vi)
        seq = self._vseq.get(key)
        ctx = s.tokens + chain
        if seq is None:
            seq = self._vseq[key] = eng.seqs.create_sequence()
        have = eng.seqs.num_tokens(seq)
        # keep the committed prefix, recompute the rest (chains are short)
        keep = min(have, len(s.tokens) - 1)
        eng.seqs.truncate(seq, keep)
        out = self._plain_prefill(eng, seq, ctx, keep)
        return torch.softmax(out[0].float() if not isinstance(out, tuple) else out[0][0].float(), -1)

    def _round(self, active, max_tokens):
        t0 = time.perf_counter()
        trees, fed = [], []
        for s in active:
            tr = DraftTree(s.tokens[-1], [DraftNode(s.tokens[-1], 1.0, 0, None, 1.0)])
            chain = []
            for _ in range(self.k):
                ds = [self._voter_dists(vi, v, s, chain) for vi, v in enumerate(self.voters)]
                j = jsd(ds)
                self.jsd_history.append(j)
                if j > self.epsilon:
                    break
                m = torch.stack(ds).mean(0)
                tok = int(m.argmax())
                tr.nodes.append(DraftNode(tok, float(m[tok]), len(chain) + 1, len(tr.nodes) - 1, 1.0))
                chain.append(tok)
            trees.append(tr)
            fed.append(set())
        t1 = time.perf_counter()
        self._verify_commit(active, trees, fed, max_tokens)
        self.stats.rounds += 1
        self.stats.draft_ms += (t1 - t0) * 1e3
        self.stats.verify_ms += (time.perf_counter() - t1) * 1e3

    def generate_batch(self, prompts, max_tokens, add_bos=True, temperature=0.0, seed=0):
        d, self.d = self.d, None           # voters keep their own sequences
        try:
            return super().generate_batch(prompts, max_tokens, add_bos, temperature, seed)
        finally:
            self.d = d
            for (sid, vi), seq in self._vseq.items():
                self.voters[vi].seqs.free_sequence(seq)
            self._vseq.clear()
