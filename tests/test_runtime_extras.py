"""Engine configuration (AIR_ env overrides), tracing spans, the expert VRAM scheduler
(reference src/moe.rs:345-504 and its tests), and KV session snapshots."""
import json

import pytest
import torch

from air_rs.config import EngineConfig
from air_rs.runtime.expert_cache import ExpertVramScheduler
from air_rs.utils import trace


# ---------------------------------------------------------------- config
def test_engine_config_defaults_and_env():
    c = EngineConfig()
    assert c.block_size == 16 and c.max_num_seqs == 256 and c.prefill_chunk == 2048
    c = EngineConfig.from_env({"AIR_MAX_BATCH": "128", "AIR_PREFIX_CACHE": "yes", "AIR_VRAM_FRACTION": "0.5",
                               "AIR_NUM_BLOCKS": "none", "AIR_CUDA_GRAPH_BATCH_SIZES": "1,2,8",
                               "AIR_PRESET": "tiny", "AIR_EXPERT_SLOTS": "4"}, tp=2)
    assert c.max_batch == 128 and c.prefix_cache is True and c.vram_fraction == 0.5
    assert c.num_blocks is None and c.cuda_graph_batch_sizes == (1, 2, 8) and c.tp == 2
    assert c.preset == "tiny" and c.expert_slots == 4
    assert json.loads(json.dumps(c.to_dict()))["max_batch"] == 128


@pytest.mark.parametrize("env", [{"AIR_BLOCK_SIZE": "12"}, {"AIR_PREFIX_CACHE": "maybe"},
                                 {"AIR_TP": "0"}, {"AIR_ALLREDUCE": "tcp"}, {"AIR_VRAM_FRACTION": "1.5"}])
def test_engine_config_rejects_bad_values(env):
    with pytest.raises(ValueError):
        EngineConfig.from_env(env)


def test_engine_config_builds_cpu_oracle_engine(tmp_path):
    from air_rs.gguf import GGMLType
    from air_rs.models.random_init import write_random_gguf
    from air_rs.models.config import tiny_llama
    p = tmp_path / "m.gguf"
    write_random_gguf(str(p), tiny_llama(), GGMLType.Q8_0, seed=0)
    eng = EngineConfig(model=str(p), device="cpu").build()
    out = eng.generate_ids([[5, 6, 7]], __import__("air_rs.runtime.engine", fromlist=["x"]).SamplingParams(
        max_tokens=3, temperature=0.0, ignore_eos=True))
    assert len(out[0]) == 3


# ---------------------------------------------------------------- tracing
def test_trace_spans_and_chrome_export(tmp_path):
    trace.clear()
    trace.enable(True)
    try:
        with trace.span("outer"):
            with trace.span("inner"):
                pass

        @trace.traced("fn")
        def f(x):
            return x + 1
        assert f(1) == 2
    finally:
        trace.enable(False)
    names = [s.name for s in trace.spans()]
    assert names.count("inner") == 1 and "outer" in names and "fn" in names
    depth = {s.name: s.depth for s in trace.spans()}
    assert depth["inner"] == depth["outer"] + 1
    summ = trace.summary()
    assert summ["outer"]["count"] == 1 and summ["outer"]["total_ms"] >= summ["inner"]["total_ms"]
    path = trace.dump_chrome(str(tmp_path / "t.json"))
    ev = json.load(open(path))["traceEvents"]
    assert {e["name"] for e in ev} >= {"outer", "inner", "fn"} and all(e["ph"] == "X" for e in ev)
    # off: nothing recorded
    trace.clear()
    with trace.span("off"):
        pass
    assert trace.spans() == []


def test_trace_engine_step_spans_cpu(tmp_path):
    from air_rs.gguf import GGMLType
    from air_rs.models.random_init import write_random_gguf
    from air_rs.models.config import tiny_llama
    from air_rs.runtime.builder import engine_from_gguf
    from air_rs.runtime.engine import SamplingParams
    p = tmp_path / "m.gguf"
    write_random_gguf(str(p), tiny_llama(), GGMLType.Q8_0, seed=0)
    eng = engine_from_gguf(str(p), device="cpu")
    trace.clear()
    trace.enable(True)
    try:
        eng.generate_ids([[1, 2, 3]], SamplingParams(max_tokens=2, temperature=0.0, ignore_eos=True))
    finally:
        trace.enable(False)
    assert any(s.name == "cpu_step" for s in trace.spans())


# ---------------------------------------------------------------- expert scheduler
def test_expert_scheduler_lru_hits_and_evictions():
    s = ExpertVramScheduler(2)
    loads = []

    def load(eid, freed):
        loads.append((eid, freed))
        return f"w{eid}"
    s.ensure_resident([0, 1], load)
    assert s.load_count == 2 and s.hit_count == 0 and s.resident_count() == 2
    s.ensure_resident([0], load)                  # hit; 1 becomes LRU
    assert s.hit_count == 1
    s.ensure_resident([2], load)                  # evicts 1, reuses its payload
    assert s.eviction_count == 1 and not s.is_resident(1) and s.is_resident(0)
    assert loads[-1] == (2, "w1")
    assert s.get(2) == "w2"
    with pytest.raises(KeyError):
        s.get(1)
    assert abs(s.hit_rate() - 1 / 4) < 1e-9
    # the experts needed together are never evicted by one another
    s.ensure_resident([1, 2], load)
    assert s.is_resident(1) and s.is_resident(2) and not s.is_resident(0)
    with pytest.raises(RuntimeError):
        s.ensure_resident([0, 1, 2], load)
    s.reset_stats()
    assert s.load_count == s.hit_count == s.eviction_count == 0


def test_expert_scheduler_prefetch_hints_by_frequency():
    s = ExpertVramScheduler(1)
    for eid in [3, 3, 3, 5, 5, 7, 1]:
        s.ensure_resident([eid], lambda e, f: e)
    # resident: 1; by use count: 3 (3x), 5 (2x), 7 (1x)
    assert s.prefetch_hints(2) == [3, 5]
    assert 1 not in s.prefetch_hints(10)
    with pytest.raises(ValueError):
        ExpertVramScheduler(0)


def test_expert_scheduler_load_failure_is_reported():
    s = ExpertVramScheduler(2)

    def bad(eid, freed):
        raise OSError("disk gone")
    with pytest.raises(RuntimeError, match="expert 4"):
        s.ensure_resident([4], bad)
    assert s.resident_count() == 0


# ---------------------------------------------------------------- KV snapshots
def _pool(L=2, nb=12, nkv=2, bs=4, d=8):
    from air_rs import _host
    kv = torch.zeros(L, nb, 2, nkv, bs, d, dtype=torch.bfloat16)
    return kv, _host.SequenceManager(nb, bs)


def test_kv_snapshot_roundtrip_bit_exact(tmp_path):
    from air_rs.kv import snapshot
    kv, seqs = _pool()
    s = seqs.create_sequence()
    seqs.append(s, 10)
    blocks = list(seqs.block_table(s))
    g = torch.Generator().manual_seed(0)
    for b in blocks:
        kv[:, b] = torch.randn(kv[:, b].shape, generator=g).bfloat16()
    toks = list(range(100, 110))
    info = snapshot.save(tmp_path / "s.kv", kv, blocks, toks)
    assert info.n_blocks == 3 and info.tokens == toks
    # a second pool with other blocks in use
    kv2, seqs2 = _pool()
    other = seqs2.create_sequence()
    seqs2.append(other, 8)
    seq, t2, b2 = snapshot.load_into(tmp_path / "s.kv", kv2, seqs2)
    assert t2 == toks and len(b2) == 3 and not set(b2) & set(seqs2.block_table(other))
    for a, b in zip(blocks, b2):
        assert torch.equal(kv[:, a], kv2[:, b])


def test_kv_snapshot_rejects_corrupt_and_foreign(tmp_path):
    from air_rs.kv import snapshot
    kv, seqs = _pool()
    s = seqs.create_sequence()
    seqs.append(s, 5)
    kv.fill_(1.0)
    snapshot.save(tmp_path / "s.kv", kv, list(seqs.block_table(s)), [1, 2, 3, 4, 5])
    p = snapshot.read(tmp_path / "s.kv")
    p["kv"].view(-1)[0] = 7.0                       # corrupt the payload, keep the header
    torch.save(p, tmp_path / "bad.kv")
    kv2, seqs2 = _pool()
    free0 = seqs2.allocator.num_free_blocks()
    with pytest.raises(snapshot.SnapshotError, match="checksum"):
        snapshot.load_into(tmp_path / "bad.kv", kv2, seqs2)
    kv3, seqs3 = _pool(d=16)                        # other geometry
    with pytest.raises(snapshot.SnapshotError, match="geometry"):
        snapshot.load_into(tmp_path / "s.kv", kv3, seqs3)
    (tmp_path / "junk.kv").write_bytes(b"not a snapshot")
    with pytest.raises(snapshot.SnapshotError):
        snapshot.read(tmp_path / "junk.kv")
    assert seqs2.allocator.num_free_blocks() == free0     # nothing allocated on failure
    with pytest.raises(snapshot.SnapshotError):
        snapshot.save(tmp_path / "x.kv", kv, [0], list(range(9)))   # 9 tokens need 3 blocks


# ---------------------------------------------------------------- GPU paths
@pytest.mark.gpu
def test_expert_cache_matches_resident_moe():
    from air_rs.gguf import GGMLType
    from air_rs.models.config import tiny_moe
    from air_rs.models.random_init import random_tensors
    from air_rs.runtime.builder import build_runner
    from air_rs.runtime.engine import Engine, SamplingParams
    cfg = tiny_moe()
    recs = list(random_tensors(cfg, GGMLType.Q4_K, seed=1, device="cpu"))
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, cfg.vocab_size, (int(n),), generator=g).tolist() for n in (20, 9, 14)]
    sp = SamplingParams(max_tokens=8, temperature=0.0, ignore_eos=True)
    outs = {}
    for slots in (None, 2):
        rn = build_runner(cfg, iter(recs), device="cuda", max_batch=16, max_model_len=256, num_blocks=256,
                          expert_slots=slots)
        eng = Engine(cfg, rn, max_batch=16)
        outs[slots] = eng.generate_ids(prompts, sp)
        rn.check_errors()
        if slots:
            st = rn.expert_cache.stats()
            assert st["loads"] > 0 and st["resident"] <= 2 and st["bytes_h2d"] > 0
            assert not any(e.data.is_cuda for lw in rn.w.layers for e in lw.experts_gu)
    assert outs[None] == outs[2]


@pytest.mark.gpu
def test_engine_snapshot_restore_hits_prefix_cache(tmp_path):
    from air_rs.runtime.builder import random_engine
    from air_rs.runtime.engine import SamplingParams
    eng = random_engine("tiny", max_batch=4, max_model_len=512, num_blocks=128, prefix_cache=True)
    prompt = list(range(3, 70))
    rid = eng.add_request(prompt, SamplingParams(max_tokens=40, temperature=0.0, ignore_eos=True))
    for _ in range(5):
        eng.step()
    st = eng.stats()
    assert st["decode_step_device_ms"] > 0 and st["kv_blocks_used"] > 0 and st["running"] == 1
    info = eng.snapshot_request(rid, tmp_path / "r.kv")
    assert info.n_blocks >= 4
    ref = eng.generate_ids([prompt], SamplingParams(max_tokens=6, temperature=0.0, ignore_eos=True))
    # a fresh engine: restore, then the same prompt reuses the restored blocks
    eng2 = random_engine("tiny", max_batch=4, max_model_len=512, num_blocks=128, prefix_cache=True)
    n = eng2.restore_snapshot(tmp_path / "r.kv")
    assert n >= 64
    out = eng2.generate_ids([prompt], SamplingParams(max_tokens=6, temperature=0.0, ignore_eos=True))
    assert eng2.prefix_cache.stats().hit_tokens >= 64
    assert out == ref


# ---------------------------------------------------------------- collective accounting
def test_comm_stats_record_capture_and_replay(tmp_path):
    import torch.distributed as dist
    from air_rs.parallel.tp import COMM, CommStats, TPGroup
    s = CommStats()
    s.record("all_reduce", 100)
    snap = s.snapshot()
    s.record("all_reduce", 50)
    s.record("peer_push", 8, calls=2)
    d = s.since(snap)
    assert d == {"all_reduce": (1, 50), "peer_push": (2, 8)}
    s.add(d, sign=-1)                       # undo a capture ...
    assert s.snapshot() == snap
    s.add(d)                                # ... and add it once per replay
    s.add(d)
    assert s.totals() == (1 + 2 + 4, 100 + 100 + 16)
    store = dist.FileStore(str(tmp_path / "fs"), 1)
    dist.init_process_group("gloo", store=store, rank=0, world_size=1)
    try:
        COMM.reset()
        tp = TPGroup()
        x = torch.zeros(2, 8)
        tp.all_reduce_add(torch.ones(2, 8), x)
        full = torch.zeros(2, 10)
        tp.all_gather_vocab(torch.ones(2, 10), full)
        assert COMM.snapshot() == {"all_reduce": (1, 64), "all_gather": (1, 80)}
    finally:
        dist.destroy_process_group()
        COMM.reset()
