"""Property-based checks of the native paged-KV bookkeeping: random sequences of create /
append / fork / truncate / swap / free keep reference counts, free-block counts and block
tables consistent with a simple Python model (small shapes, many operations)."""
from collections import Counter

from hypothesis import given, settings, strategies as st

from air_rs import _host

BLOCKS, BS = 24, 4


def _check(m, live, swapped):
    alloc = m.allocator
    refs = Counter()
    for s in live:
        if s in swapped:
            continue
        tab = list(m.block_table(s))
        assert len(tab) == -(-m.num_tokens(s) // BS)
        refs.update(tab)
    for b, n in refs.items():
        assert alloc.ref_count(b) == n, (b, n, alloc.ref_count(b))
    assert alloc.num_used_blocks() == len(refs)
    assert alloc.num_free_blocks() == BLOCKS - len(refs)


ops = st.lists(st.tuples(st.sampled_from(["create", "append", "fork", "truncate", "swap", "swapin", "free"]),
                         st.integers(0, 7), st.integers(1, 13)), min_size=1, max_size=60)


@settings(max_examples=200, deadline=None)
@given(ops)
def test_random_operations_keep_invariants(seq_ops):
    m = _host.SequenceManager(BLOCKS, BS)
    live, swapped = [], set()
    for op, pick, n in seq_ops:
        cur = [s for s in live if s not in swapped]
        try:
            if op == "create":
                live.append(m.create_sequence())
            elif op == "append" and cur:
                s = cur[pick % len(cur)]
                need = -(-(m.num_tokens(s) + n) // BS) - -(-m.num_tokens(s) // BS)
                if m.allocator.can_allocate(need):
                    m.append(s, n)
            elif op == "fork" and cur:
                live.append(m.fork_sequence(cur[pick % len(cur)]))
            elif op == "truncate" and cur:
                s = cur[pick % len(cur)]
                m.truncate(s, min(m.num_tokens(s), n))
            elif op == "swap" and cur:
                s = cur[pick % len(cur)]
                m.swap_out(s)
                swapped.add(s)
            elif op == "swapin" and swapped:
                s = sorted(swapped)[pick % len(swapped)]
                if m.allocator.can_allocate(-(-m.num_tokens(s) // BS)):
                    m.swap_in(s)
                    swapped.discard(s)
            elif op == "free" and live:
                s = live.pop(pick % len(live))
                m.free_sequence(s)
                swapped.discard(s)
        except (RuntimeError, ValueError, IndexError):
            pass        # refused operations (pool exhausted) must leave the state intact
        _check(m, live, swapped)
    for s in list(live):
        m.free_sequence(s)
    assert m.allocator.num_free_blocks() == BLOCKS


prefix_ops = st.lists(st.tuples(st.sampled_from(["insert", "match", "evict", "finish"]),
                                st.lists(st.integers(0, 2), min_size=1, max_size=12), st.integers(0, 5)),
                      min_size=1, max_size=40)


@settings(max_examples=150, deadline=None)
@given(prefix_ops)
def test_prefix_cache_refcounts(seq_ops):
    """Cached blocks hold one reference each; a match returns a real prefix of an inserted
    prompt; eviction frees only blocks no live sequence uses."""
    from air_rs.kv.prefix_cache import RadixCache
    m = _host.SequenceManager(BLOCKS, BS)
    cache = RadixCache(BS, 8, m.allocator)
    live, inserted = [], []
    for op, toks, k in seq_ops:
        toks = [t for t in toks for _ in range(2)]          # 2-24 tokens over a tiny alphabet
        if op == "insert":
            need = -(-len(toks) // BS)
            if not m.allocator.can_allocate(need):
                continue
            s = m.create_sequence()
            m.append(s, len(toks))
            cache.insert(toks, list(m.block_table(s)))
            live.append(s)
            inserted.append(toks)
        elif op == "match":
            n, blocks = cache.longest_prefix_match(toks)
            assert n == len(blocks) * BS and n <= len(toks)
            if n:
                assert any(p[:n] == toks[:n] for p in inserted)
        elif op == "evict":
            cache.evict_until(k)
        elif op == "finish" and live:
            m.free_sequence(live.pop(k % len(live)))
        # every cached block is held by the cache; blocks of live sequences by them too
        held = Counter()
        for s in live:
            held.update(m.block_table(s))
        stack = list(cache._roots.values())
        while stack:
            node = stack.pop()
            for c in node.children.values():
                held[c.block] += 1
                stack.append(c)
        for b, n in held.items():
            assert m.allocator.ref_count(b) == n
        assert m.allocator.num_used_blocks() == len(held)
    cache.clear()
    for s in live:
        m.free_sequence(s)
    assert m.allocator.num_free_blocks() == BLOCKS
