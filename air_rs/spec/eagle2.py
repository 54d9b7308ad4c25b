"""EAGLE-2 style draft trees (reference ``src/eagle2.rs``).

Constants are the reference's: depth <= 6, expand a node only if its draft probability is
at least tau = 0.05, top-4 children per expanded node. ``DraftTree`` stores nodes in BFS
order with their parent, depth and draft probability; ``to_mask`` is the ancestor mask used
by tree attention (node i attends to node j iff j is i or an ancestor of i).

``Eagle2Builder`` here expands the tree one *level* at a time (all frontier nodes of a depth
in one draft forward) instead of one full draft forward per node as the reference does
(``src/speculative.rs:255-263``); the resulting tree is the same.

``accept_sample`` is speculative sampling: accept draft token x with probability
min(1, p(x)/q(x)); on rejection draw from the residual max(0, p - q) (normalised), which
keeps the output distribution exactly the target's.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Protocol

import torch

MAX_TREE_DEPTH = 6
EXPAND_THRESHOLD = 0.05
DRAFT_TOP_K = 4
MAX_TREE_NODES = 64          # tree attention carries one 64-bit ancestor mask per node


@dataclass
class DraftNode:
    token_id: int
    draft_prob: float
    depth: int
    parent_idx: int | None
    cum_prob: float = 1.0


@dataclass
class DraftTree:
    root_token: int
    nodes: list[DraftNode] = field(default_factory=list)

    def __len__(self):
        return len(self.nodes)

    def children(self, idx: int | None) -> list[int]:
        return [i for i, n in enumerate(self.nodes) if n.parent_idx == idx]

    def path_to_root(self, idx: int) -> list[int]:
        out = []
        while idx is not None:
            out.append(idx)
            idx = self.nodes[idx].parent_idx
        return out[::-1]

    def all_paths(self) -> list[list[int]]:
        leaves = [i for i in range(len(self.nodes)) if not self.children(i)]
        return [self.path_to_root(i) for i in leaves]

    def flatten(self) -> list[int]:
        return [n.token_id for n in self.nodes]

    def to_mask(self) -> torch.Tensor:
        n = len(self.nodes)
        m = torch.zeros(n, n, dtype=torch.bool)
        for i in range(n):
            for j in self.path_to_root(i):
                m[i, j] = True
        return m

    def ancestor_bits(self, offset: int = 0) -> list[int]:
        """Per node: bitmask over (offset + node index) of itself and its ancestors."""
        out = []
        for i in range(len(self.nodes)):
            b = 0
            for j in self.path_to_root(i):
                b |= 1 << (offset + j)
            out.append(b)
        return out


class DraftModel(Protocol):
    def next_logits(self, context: list[int]) -> torch.Tensor: ...


def _topk(probs: torch.Tensor, k: int):
    v, i = torch.topk(probs, min(k, probs.numel()))
    return list(zip(i.tolist(), v.tolist()))


class Eagle2Builder:
    def __init__(self, draft: DraftModel | None = None, tau: float = EXPAND_THRESHOLD, top_k: int = DRAFT_TOP_K,
                 max_depth: int = MAX_TREE_DEPTH, max_nodes: int = MAX_TREE_NODES):
        self.draft, self.tau, self.top_k, self.max_depth, self.max_nodes = draft, tau, top_k, max_depth, max_nodes

    def expand_level(self, tree: DraftTree, frontier: list[int | None], probs: list[torch.Tensor]) -> list[int]:
        """Add top-k children under each frontier node; returns the next frontier."""
        nxt = []
        for parent, p in zip(frontier, probs):
            nxt.extend(self.add_children(tree, parent, _topk(p, self.top_k)))
        return nxt

    def add_children(self, tree: DraftTree, parent: int | None, cands: list[tuple[int, float]]) -> list[int]:
        """Append (token, draft prob) children, best first; returns those to expand further."""
        nxt = []
        depth = 0 if parent is None else tree.nodes[parent].depth + 1
        base = 1.0 if parent is None else tree.nodes[parent].cum_prob
        for tok, q in cands[: self.top_k]:
            if len(tree.nodes) >= self.max_nodes:
                break
            tree.nodes.append(DraftNode(tok, q, depth, parent, base * q))
            if q >= self.tau and depth + 1 < self.max_depth:
                nxt.append(len(tree.nodes) - 1)
        return nxt

    def build(self, context: list[int]) -> DraftTree:
        """Reference-equivalent BFS using ``DraftModel.next_logits`` (one call per node)."""
        tree = DraftTree(context[-1] if context else 0)
        frontier: list[int | None] = [None]
        while frontier:
            probs = []
            for f in frontier:
                ctx = list(context) + ([] if f is None else [tree.nodes[j].token_id for j in tree.path_to_root(f)])
                probs.append(torch.softmax(self.draft.next_logits(ctx).float(), -1))
            frontier = self.expand_level(tree, frontier, probs)
        return tree


@dataclass
class VerificationResult:
    n_accepted: int
    bonus_token: int
    path: list[int]


def accept_sample(path: list[int], target_probs: list[torch.Tensor], draft_probs: list,
                  rng: Callable[[], float]) -> VerificationResult:
    """Speculative sampling along one path. ``draft_probs[i]`` is q(path[i]) (scalar) or the
    full draft distribution at that position (tensor), used for the exact residual."""
    assert len(path) == len(target_probs) == len(draft_probs)
    for i, (tok, p) in enumerate(zip(path, target_probs)):
        q = draft_probs[i]
        q_tok = float(q[tok]) if isinstance(q, torch.Tensor) else float(q)
        if rng() < min(1.0, float(p[tok]) / max(q_tok, 1e-8)):
            continue
        if isinstance(q, torch.Tensor):
            resid = (p - q).clamp_min(0.0)
        else:
            resid = p.clone()
            resid[tok] = max(0.0, float(p[tok]) - q_tok)
        s = float(resid.sum())
        if s < 1e-8:
            bonus = int(torch.argmax(p))
        else:
            c = torch.cumsum(resid / s, 0)
            bonus = int(torch.searchsorted(c, torch.tensor(rng())).clamp(max=p.numel() - 1))
        return VerificationResult(i, bonus, path)
    # all accepted: the caller samples the bonus from the next position's target distribution
    return VerificationResult(len(path), -1, path)


def greedy_accept(tree: DraftTree, target_next: list[int]) -> tuple[list[int], int]:
    """Greedy verification over a tree whose node 0 is the root (the pending token).

    ``target_next[i]`` is the target's argmax after node i. Returns (accepted node indices
    starting with 0, bonus token)."""
    path = [0]
    while True:
        want = target_next[path[-1]]
        nxt = [c for c in tree.children(path[-1]) if tree.nodes[c].token_id == want]
        if not nxt:
            return path, want
        path.append(nxt[0])
