"""Scheduling policies: ARB, Orca/Sarathi continuous batching, batch optimiser, ModelMux
(reference tests in src/batching/arb.rs, src/continuous_batch.rs, src/batch_optimizer.rs,
src/model_mux.rs)."""
import time

import pytest

from air_rs.sched.arb import (ArbConfig, ArbScheduler, ContinuousBatchScheduler, HarmonicGroup, KvSlotAllocator,
                              Phase, Priority)
from air_rs.sched.batch_optimizer import ComputeProfile, StorageProfile, optimal_batch


def test_harmonic_group_ratio():
    g = HarmonicGroup([0], 100, 100)
    assert g.can_admit(150, 2.0) and g.can_admit(50, 2.0) and not g.can_admit(201, 2.0)


def test_slot_allocator():
    a = KvSlotAllocator(2)
    s0, s1 = a.alloc(), a.alloc()
    assert a.alloc() is None and a.available() == 0
    a.free(s0)
    assert a.alloc() == s0
    with pytest.raises(ValueError):
        a.free(7)


def test_arb_groups_by_length_prefills_in_chunks_and_coasts():
    cfg = ArbConfig(kv_slots=8, prefill_chunk_size=4, confidence_exit_k=2, coast_ms=1000)
    s = ArbScheduler(cfg)
    short = [s.enqueue([1] * 10, urgency=1.0) for _ in range(2)]
    long_ = s.enqueue([2] * 100)
    s.admit_waiting()
    b = s.build_micro_batch()
    ids = {e.seq_id for e in b}
    assert ids == set(short)                         # 10 vs 100 tokens: different harmonic groups
    assert all(e.phase == Phase.PREFILL and len(e.tokens) == 4 for e in b)
    for _ in range(3):                               # 3 chunks of 4 cover the 10-token prompts
        s.commit_results([(e.seq_id, 5, 0.5, False) for e in s.build_micro_batch() if e.seq_id in short])
    assert all(s.active[i].phase == Phase.DECODE for i in short)
    for _ in range(2):
        s.commit_results([(i, 6, 0.99, False) for i in short])
    assert all(s.active[i].phase == Phase.COASTING for i in short)
    b = s.build_micro_batch()
    assert {e.seq_id for e in b} == {long_}          # coasting sequences yield the batch
    s.commit_results([(short[0], 0, 0.1, True)])
    assert short[0] not in s.active and s.alloc.available() == 8 - 2


def test_continuous_batch_budget_and_priority():
    cb = ContinuousBatchScheduler(max_batch=4, token_budget=20, chunk=8)
    a = cb.submit(30, 2)
    b = cb.submit(5, 2, Priority.HIGH)
    sb = cb.schedule()
    assert sb.decode == [] and sb.prefill == [(b, 0, 5), (a, 0, 8)] and sb.num_tokens == 13
    cb.prefill_done(b, 5)
    cb.prefill_done(a, 8)
    sb = cb.schedule()
    assert sb.decode == [b] and sb.prefill == [(a, 8, 8)]
    assert cb.decode_step([b]) == [b] and cb.abort(a)


def test_batch_optimizer_regimes():
    r = optimal_batch(8e9, 0.5625, 131072, 2048, 100 << 30)
    assert r.bound == "compute" and 16 < r.batch < 1024
    r2 = optimal_batch(8e9, 0.5625, 131072, 2048, 2 << 30)
    assert r2.bound == "kv" and r2.batch == (2 << 30) // (131072 * 2048)
    r3 = optimal_batch(8e9, 0.5625, 131072, 2048, 100 << 30, storage=StorageProfile(resident=False))
    assert r3.batch > r.batch and r3.tokens_per_s < r.tokens_per_s


def test_model_mux_round_robin_on_cpu_engines():
    from air_rs.gguf import GGMLType
    from air_rs.models.config import tiny_llama
    from air_rs.models.random_init import random_tensors
    from air_rs.models.reference import OracleModel
    from air_rs.runtime.engine import Engine, SamplingParams
    from air_rs.sched.mux import ModelMux, MuxEventKind
    cfg = tiny_llama()
    mux = ModelMux()
    for name, seed in (("a", 0), ("b", 1)):
        recs = list(random_tensors(cfg, GGMLType.Q8_0, seed=seed, device="cpu"))
        mux.add_model(name, Engine(cfg, None, oracle=OracleModel(cfg, {n: (r, q, s) for n, r, q, s in recs})))
    sp = SamplingParams(max_tokens=3, temperature=0.0, ignore_eos=True)
    ra, rb = mux.submit("a", [5, 6], sp), mux.submit("b", [7, 8], sp)
    mux.run_until_idle()
    fin = [(e.model, e.rid) for e in mux.events if e.kind == MuxEventKind.FINISHED]
    assert sorted(fin) == [("a", ra), ("b", rb)]
    toks = [e.model for e in mux.events if e.kind == MuxEventKind.TOKEN]
    assert toks[:2] == ["a", "b"] and len(toks) == 6


def test_engine_admission_policies():
    import time as _t
    from air_rs.models.config import tiny_llama
    from air_rs.runtime.engine import Engine, Request, SamplingParams
    cfg = tiny_llama()
    sp = SamplingParams()
    mk = lambda rid, n, pr=0: Request(rid, list(range(n)), sp, priority=pr)
    e = Engine(cfg, None, admission="priority")
    e.waiting.extend([mk(0, 10), mk(1, 10, pr=5), mk(2, 10, pr=5)])
    assert e._next_waiting([]).rid == 1
    a = Engine(cfg, None, admission="arb", arb_ratio=2.0, max_wait_s=60.0)
    a.running = [mk(9, 100)]
    a.waiting.extend([mk(0, 1000), mk(1, 20), mk(2, 150)])
    assert a._next_waiting([]).rid == 2            # within 2x of the running context
    a.waiting[0].arrival = _t.perf_counter() - 120  # starving: goes first
    assert a._next_waiting([]).rid == 0
    f = Engine(cfg, None)
    f.waiting.extend([mk(0, 5), mk(1, 5, pr=9)])
    assert f._next_waiting([]).rid == 0
    import pytest
    with pytest.raises(ValueError):
        Engine(cfg, None, admission="lifo")
