"""Radix prefix cache over paged KV blocks (reference ``src/prefix_cache.rs``: RadixCache with
LRU/LFU eviction, tenant isolation, pinning, hit statistics).

The reference keeps token ids -> block ids in a Patricia trie that nothing consults. Here
the trie is block-granular (an edge is the token ids of one full KV block) and owns a
reference on every block it stores (``BlockAllocator.share``), so a cached prefix stays in
HBM after its request finishes; a new request whose prompt starts with a cached prefix gets
those blocks in its block table (``SequenceManager.create_with_prefix``) and only prefills
the rest. Partially filled blocks are never cached, so cached blocks are immutable.
"""
from __future__ import annotations

import enum
import itertools
from dataclasses import dataclass, field


class EvictionPolicy(str, enum.Enum):
    LRU = "lru"
    LFU = "lfu"


@dataclass
class PrefixCacheStats:
    lookups: int = 0
    hits: int = 0
    hit_tokens: int = 0
    inserted_blocks: int = 0
    evicted_blocks: int = 0
    cached_blocks: int = 0

    @property
    def hit_rate(self) -> float:
        return self.hits / self.lookups if self.lookups else 0.0


@dataclass(eq=False)
class _Node:
    key: tuple = ()
    block: int = -1
    parent: "_Node | None" = None
    children: dict = field(default_factory=dict)
    last_use: int = 0
    uses: int = 0
    pinned: int = 0


class RadixCache:
    """Block-granular radix cache. ``allocator`` is the engine's ``BlockAllocator`` (share /
    release / ref_count); with ``allocator=None`` it is pure bookkeeping (tests)."""

    def __init__(self, block_size: int, max_blocks: int, allocator=None,
                 eviction_policy: EvictionPolicy = EvictionPolicy.LRU):
        self.block_size = block_size
        self.max_blocks = max_blocks
        self.alloc = allocator
        self.policy = EvictionPolicy(eviction_policy)
        self._roots: dict[str | None, _Node] = {}
        self._clock = itertools.count(1)
        self.stats_ = PrefixCacheStats()

    # ------------------------------------------------------------------ lookup
    def _root(self, tenant):
        r = self._roots.get(tenant)
        if r is None:
            r = self._roots[tenant] = _Node()
        return r

    def _chunks(self, tokens):
        bs = self.block_size
        for i in range(len(tokens) // bs):
            yield tuple(tokens[i * bs:(i + 1) * bs])

    def longest_prefix_match_for_tenant(self, tokens, tenant_id: str | None = None,
                                        max_tokens: int | None = None) -> tuple[int, list[int]]:
        """(matched token count, block ids) of the longest cached whole-block prefix."""
        self.stats_.lookups += 1
        node = self._roots.get(tenant_id)
        blocks: list[int] = []
        limit = len(tokens) if max_tokens is None else min(len(tokens), max_tokens)
        if node is not None:
            now = next(self._clock)
            for key in self._chunks(tokens[:limit]):
                nxt = node.children.get(key)
                if nxt is None:
                    break
                nxt.last_use = now
                nxt.uses += 1
                blocks.append(nxt.block)
                node = nxt
        n = len(blocks) * self.block_size
        if blocks:
            self.stats_.hits += 1
            self.stats_.hit_tokens += n
        return n, blocks

    def longest_prefix_match(self, tokens, max_tokens: int | None = None):
        return self.longest_prefix_match_for_tenant(tokens, None, max_tokens)

    # ------------------------------------------------------------------ insert / evict
    def insert_for_tenant(self, tokens, kv_block_ids, tenant_id: str | None = None) -> int:
        """Cache the whole blocks of ``tokens`` (kv_block_ids[i] holds block i). Returns the
        number of blocks newly cached."""
        node = self._root(tenant_id)
        now = next(self._clock)
        added = 0
        for i, key in enumerate(self._chunks(tokens)):
            if i >= len(kv_block_ids):
                break
            nxt = node.children.get(key)
            if nxt is None:
                if self.size() >= self.max_blocks and self.evict_until(1, protect=node) == 0:
                    break
                nxt = _Node(key, int(kv_block_ids[i]), node)
                node.children[key] = nxt
                if self.alloc is not None:
                    self.alloc.share(nxt.block)
                added += 1
            nxt.last_use = now
            node = nxt
        self.stats_.inserted_blocks += added
        return added

    def insert(self, tokens, kv_block_ids) -> int:
        return self.insert_for_tenant(tokens, kv_block_ids, None)

    def _leaves(self):
        stack = list(self._roots.values())
        while stack:
            n = stack.pop()
            if n.children:
                stack.extend(n.children.values())
            elif n.parent is not None:
                yield n

    def _evictable(self, n: _Node) -> bool:
        if n.pinned:
            return False
        # a block still used by a live sequence is not freed by evicting it; skip it
        return self.alloc is None or self.alloc.ref_count(n.block) <= 1

    def evict_until(self, free_target: int, protect: _Node | None = None) -> int:
        """Drop up to ``free_target`` cached leaf blocks (LRU or LFU order); returns how many."""
        freed = 0
        while freed < free_target:
            cands = [n for n in self._leaves() if n is not protect and self._evictable(n)]
            if not cands:
                break
            key = (lambda n: (n.last_use,)) if self.policy == EvictionPolicy.LRU else (lambda n: (n.uses, n.last_use))
            victim = min(cands, key=key)
            del victim.parent.children[victim.key]
            if self.alloc is not None:
                self.alloc.release(victim.block)
            freed += 1
        self.stats_.evicted_blocks += freed
        return freed

    def pin(self, tokens, tenant_id: str | None = None):
        self._set_pin(tokens, tenant_id, +1)

    def unpin(self, tokens, tenant_id: str | None = None):
        self._set_pin(tokens, tenant_id, -1)

    def _set_pin(self, tokens, tenant, d):
        node = self._roots.get(tenant)
        for key in self._chunks(tokens):
            if node is None:
                return
            node = node.children.get(key)
            if node is not None:
                node.pinned = max(0, node.pinned + d)

    def size(self) -> int:
        n, stack = 0, list(self._roots.values())
        while stack:
            x = stack.pop()
            n += len(x.children)
            stack.extend(x.children.values())
        return n

    def clear(self):
        self.evict_until(self.size() + 1)
        # pinned nodes remain referenced; drop them too on an explicit clear
        for r in self._roots.values():
            stack = list(r.children.values())
            while stack:
                x = stack.pop()
                stack.extend(x.children.values())
                if self.alloc is not None:
                    self.alloc.release(x.block)
            r.children.clear()

    def stats(self) -> PrefixCacheStats:
        self.stats_.cached_blocks = self.size()
        return self.stats_
