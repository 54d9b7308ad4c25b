"""KV memory management: radix prefix cache, swap to host, tier policy, VRAM guard
(reference tests in src/prefix_cache.rs, src/kv_swap.rs, src/kv_tier.rs, src/vram_guard.rs)."""
import pytest
import torch

from air_rs import _host
from air_rs.kv.prefix_cache import EvictionPolicy, RadixCache
from air_rs.kv.swap import KvSwapManager
from air_rs.kv.tiers import HermesTierManager, HermesWeights, KvTier, TierBudget, TierManager, TokenEntry
from air_rs.runtime.vram_guard import VramBudget


def _seq_with(mgr, tokens):
    s = mgr.create_sequence()
    mgr.append(s, len(tokens))
    return s


def test_radix_match_insert_and_refcounts():
    mgr = _host.SequenceManager(64, 4)
    cache = RadixCache(4, 32, mgr.allocator)
    toks = list(range(10))                       # 2 whole blocks + 2 tokens
    s = _seq_with(mgr, toks)
    blocks = mgr.block_table(s)
    assert cache.insert(toks, blocks) == 2
    assert mgr.allocator.ref_count(blocks[0]) == 2
    n, got = cache.longest_prefix_match(toks + [99, 98])
    assert n == 8 and got == blocks[:2]
    n, got = cache.longest_prefix_match([0, 1, 2, 3, 7, 7, 7, 7])
    assert n == 4 and got == blocks[:1]
    n, _ = cache.longest_prefix_match([5, 5, 5, 5])
    assert n == 0
    st = cache.stats()
    assert st.lookups == 3 and st.hits == 2 and st.cached_blocks == 2
    # a new sequence built from the prefix shares the blocks and appends past them
    s2 = mgr.create_with_prefix(got, 4)
    assert mgr.block_table(s2) == blocks[:1] and mgr.allocator.ref_count(blocks[0]) == 3
    mgr.append(s2, 1)
    assert len(mgr.block_table(s2)) == 2 and mgr.block_table(s2)[1] not in blocks
    # freeing the owners leaves the cache's reference
    mgr.free_sequence(s)
    mgr.free_sequence(s2)
    assert mgr.allocator.ref_count(blocks[0]) == 1
    assert cache.evict_until(10) == 2
    assert mgr.allocator.num_used_blocks() == 0


def test_radix_tenant_isolation_pin_and_lfu():
    cache = RadixCache(2, 3, None, EvictionPolicy.LFU)
    cache.insert_for_tenant([1, 2, 3, 4], [10, 11], "a")
    assert cache.longest_prefix_match_for_tenant([1, 2, 3, 4], "b")[0] == 0
    assert cache.longest_prefix_match_for_tenant([1, 2, 3, 4], "a") == (4, [10, 11])
    cache.insert_for_tenant([7, 7], [12], "a")
    cache.pin([7, 7], "a")
    # full (3 blocks): inserting evicts the least frequently used unpinned leaf
    cache.insert_for_tenant([9, 9], [13], "a")
    assert cache.size() == 3
    assert cache.longest_prefix_match_for_tenant([7, 7], "a")[0] == 2       # pinned survives
    assert cache.longest_prefix_match_for_tenant([1, 2, 3, 4], "a")[0] == 2  # leaf 11 was evicted


def test_swap_roundtrip_bit_exact_cpu():
    mgr = _host.SequenceManager(16, 4)
    kv = torch.randn(3, 16, 2, 2, 4, 8)
    a = _seq_with(mgr, list(range(10)))
    b = _seq_with(mgr, list(range(6)))
    before = kv[:, mgr.block_table(a)].clone()
    sw = KvSwapManager(kv, mgr)
    freed = sw.evict(a)
    assert sw.is_evicted(a) and mgr.is_swapped(a) and len(freed) == 3
    kv[:, freed] = 0.0                        # the pool reuses the blocks meanwhile
    c = _seq_with(mgr, list(range(8)))
    new = sw.restore(a)
    assert not sw.is_evicted(a) and mgr.num_tokens(a) == 10
    assert torch.equal(kv[:, new], before)
    assert not set(new) & set(mgr.block_table(c)) and not set(new) & set(mgr.block_table(b))


def test_tier_manager_budgets_and_promotion():
    tm = TierManager(TierBudget(pinned_max=2, active_max=3, warm_max=2))
    for p in range(8):
        tm.add_token(p)
    tm.pin_range(0, 2)
    tm.touch_positions([7])
    tm.enforce_budgets()
    assert tm.distribution() == (2, 3, 2, 1)
    assert tm.get_tier(2) == KvTier.COLD and tm.get_tier(7) == KvTier.ACTIVE
    assert tm.promote(2) and tm.get_tier(2) == KvTier.ACTIVE and not tm.promote(0)
    b = TierBudget.from_vram(1 << 30, 1 << 16)
    assert b.pinned_max == 3276 and b.active_max == 16384 - 3276 and b.warm_max == 4 * b.active_max


def test_hermes_prefers_prefix_and_frequent_tokens():
    w = HermesWeights()
    hot = TokenEntry(5, KvTier.ACTIVE, access_count=20, last_step=99)
    cold = TokenEntry(900, KvTier.ACTIVE, access_count=0, last_step=0)
    assert w.score(hot, 100) > w.score(cold, 100)
    hm = HermesTierManager(TierBudget(pinned_max=0, active_max=2, warm_max=10))
    for p in range(4):
        hm.add_token(p)
    hm.touch_positions([0, 0, 0])
    hm.enforce_budgets()
    assert hm.get_tier(0) == KvTier.ACTIVE and hm.count_tier(KvTier.WARM) == 2


def test_vram_guard_accept_reject_skip():
    gib = 1 << 30
    fake = lambda dev: (100 * gib, 180 * gib)
    assert VramBudget.check(100 * gib, mem_get_info=fake).ok_to_load()
    r = VramBudget.check(150 * gib, mem_get_info=fake)
    assert not r.ok_to_load() and r.shortfall_bytes == 150 * gib - int(180 * gib * 0.8)
    assert "rejected" in r.summary()

    def boom(dev):
        raise RuntimeError("no device")
    assert VramBudget.check(1, mem_get_info=boom).kind == "skipped"
    est = VramBudget.estimate(4 << 30, 32, 8, 128, 8192)
    assert est == (4 << 30) + 2 * 32 * 8 * 128 * 8192 * 2 + (512 << 20)


@pytest.mark.gpu
def test_engine_prefix_cache_and_preemption():
    from air_rs.runtime.builder import build_runner
    from air_rs.runtime.engine import Engine, SamplingParams
    from air_rs.models.config import tiny_llama
    from air_rs.models.random_init import random_tensors
    from air_rs.models.reference import OracleModel
    from air_rs.gguf import GGMLType
    from test_engine_gpu import _check_near_argmax
    cfg = tiny_llama()
    recs = list(random_tensors(cfg, GGMLType.Q8_0, seed=0, device="cpu"))
    oracle = OracleModel(cfg, {n: (r, q, s) for n, r, q, s in recs})
    g = torch.Generator().manual_seed(3)
    shared = torch.randint(0, cfg.vocab_size, (40,), generator=g).tolist()
    prompts = [shared + torch.randint(0, cfg.vocab_size, (int(n),), generator=g).tolist() for n in (5, 9, 17, 3)]
    sp = SamplingParams(max_tokens=24, temperature=0.0, repetition_penalty=1.0, ignore_eos=True)

    def engine(**kw):
        rn = build_runner(cfg, iter(recs), device="cuda", max_batch=8, max_model_len=256,
                          num_blocks=kw.pop("num_blocks", 256))
        return Engine(cfg, rn, max_batch=8, **kw)

    eng = engine(prefix_cache=True)
    out = eng.generate_ids(prompts[:1], sp) + eng.generate_ids(prompts[1:], sp)
    st = eng.prefix_cache.stats()
    assert st.hits >= 3 and st.cached_blocks >= 2
    # BOS + 40 shared tokens = two whole 16-token blocks served from the cache
    assert sorted(r.cached_tokens for r in eng.finished.values()) == [0, 32, 32, 32]
    for p, o in zip(prompts, out):
        assert len(o) == 24
        _check_near_argmax(oracle, [cfg.bos_token_id] + p, o, penalty=1.0)

    # a pool too small for all four sequences at once forces swap-out / swap-in
    sp = SamplingParams(max_tokens=64, temperature=0.0, repetition_penalty=1.0, ignore_eos=True)
    eng = engine(num_blocks=12)
    out = eng.generate_ids(prompts, sp)
    assert getattr(eng.metrics, "preemptions", 0) > 0 and eng.swap.bytes_in > 0
    for p, o in zip(prompts, out):
        assert len(o) == 64
        _check_near_argmax(oracle, [cfg.bos_token_id] + p, o, penalty=1.0)
    assert eng.seqs.allocator.num_used_blocks() == 0


def test_tri_attention_scores_match_definition():
    """TriAttention (reference src/tri_attention.rs:17-28, 93-129): sinks score 1, the rest is
    the min-max normalised blend of the scaled head-mean cosine and the RoPE phase term."""
    import math
    import torch
    from air_rs.kv.tri_attention import ALPHA, SINK_COUNT, TriScorer, TriAttentionTierManager
    from air_rs.kv.tiers import KvTier, TierBudget
    H, D, S = 4, 64, 40
    g = torch.Generator().manual_seed(0)
    q = torch.randn(H * D, generator=g)
    k = torch.randn(S, H, D, generator=g)
    sc = TriScorer(D, H, 10000.0)
    got = sc.score(q, k)
    # per-position loop, straight from the definition
    freqs = [1.0 / 10000.0 ** (2 * i / D) for i in range(D // 2)]
    raw = []
    for p in range(S):
        if p < SINK_COUNT:
            raw.append(1.0)
            continue
        sims = []
        for h in range(H):
            qh, kh = q[h * D:(h + 1) * D], k[p, h]
            c = float(qh @ kh) * D ** -0.25 / (float(qh.norm()) * float(kh.norm()))
            sims.append(max(-1.0, min(1.0, c)))
        ph = (sum(math.cos(f * p) for f in freqs) / len(freqs) + 1) / 2
        raw.append(max(0.0, min(1.0, ALPHA * sum(sims) / H + (1 - ALPHA) * ph)))
    lo, hi = min(raw[SINK_COUNT:]), max(raw[SINK_COUNT:])
    ref = raw[:SINK_COUNT] + [(r - lo) / (hi - lo) for r in raw[SINK_COUNT:]]
    torch.testing.assert_close(got, torch.tensor(ref), rtol=1e-4, atol=1e-5)
    m = TriScorer.keep_mask(got, 10)
    assert int(m.sum()) == 10 and bool(m[:SINK_COUNT].all())
    assert int(TriScorer.keep_mask(got, 1).sum()) == SINK_COUNT + 1      # minimum budget
    # as a tier manager: the lowest-scoring active positions are demoted first
    mgr = TriAttentionTierManager(TierBudget(pinned_max=4, active_max=30, warm_max=100), sc)
    for p in range(S):
        mgr.add_token(p)
    mgr.update_scores(q, k)
    mgr.enforce_budgets()
    warm = sorted(p for p, e in mgr.entries.items() if e.tier == KvTier.WARM)
    expect = sorted(sorted(range(S), key=lambda p: (float(got[p]), p))[:S - 30])
    assert warm == expect
