"""Residency scoring, priority I/O engine and residency scheduler (reference
src/strix/score.rs, io_engine.rs, scheduler.rs tests)."""
import math
import os

import pytest
import torch

from air_rs.stream import strix as S


def test_score_components():
    assert S.urgency(0, 3) > 0.9 and abs(S.urgency(3, 3) - 0.5) < 0.01 and S.urgency(10, 3) < 0.01
    assert S.urgency(0, 0) == 1.0 and S.urgency(1, 0) == 0.0
    assert S.predictive(5, 5) == 1.0 and abs(S.predictive(0, 10, 0.1) - math.exp(-1)) < 1e-9
    assert S.sticky(0) == 0.0 and abs(S.sticky(20) - 1.0) < 1e-9 and 0 < S.sticky(3) < 1
    assert S.cost(50, 100) == 0.5 and S.cost(500, 100) == 1.0 and S.cost(1, 0) == 0.0
    w = S.ScoreWeights()
    assert abs(w.sum() - 1.0) < 1e-9 and S.residency_score(w, 1, 1, 1, 1) == 1.0
    assert S.IoPriority.from_class(S.TensorClass.A, False) == S.IoPriority.CRITICAL
    assert S.IoPriority.from_class(S.TensorClass.C, True) == S.IoPriority.HIGH
    assert S.IoPriority.from_class(S.TensorClass.D, True) == S.IoPriority.LOW


def test_io_engine_reads_in_priority_order(tmp_path):
    p = tmp_path / "blob.bin"
    data = os.urandom(1 << 16)
    p.write_bytes(data)
    eng = S.IoEngine(str(p), capacity=1, workers=1, pin=False, start_paused=True)
    try:
        eng.submit(S.IoRequest("first", 0, 4096, S.IoPriority.NORMAL))
        eng.submit(S.IoRequest("low", 8192, 100, S.IoPriority.LOW))
        eng.submit(S.IoRequest("crit", 100, 1000, S.IoPriority.CRITICAL))
        eng.submit(S.IoRequest("bad", len(data) - 10, 100, S.IoPriority.HIGH))
        assert eng.queued_count() == 4
        eng.resume()
        done = eng.wait_all()
    finally:
        eng.close()
    by = {c.tensor_id: c for c in done}
    assert bytes(by["crit"].data.numpy()) == data[100:1100] and bytes(by["low"].data.numpy()) == data[8192:8292]
    assert by["bad"].error is not None and by["crit"].error is None
    order = [c.tensor_id for c in done]
    assert order == ["crit", "bad", "first", "low"]


def test_residency_scheduler_budget_and_window():
    sch = S.ResidencyScheduler(budget_bytes=300, prefetch_window=1)
    sch.register(S.TrackedTensor("embd", 100, S.TensorClass.A))
    for i in range(4):
        sch.register(S.TrackedTensor(f"l{i}", 100, S.TensorClass.B, layer=i))
    load, evict = sch.tick(current_layer=0, n_layers=4)
    assert "embd" in load and {"l0", "l1"} <= set(load) and not evict
    load, evict = sch.tick(current_layer=2, n_layers=4)
    assert {"l2", "l3"} & set(load) and evict and sch.tensors[evict[0]].evictions == 1
    resident = [t.tensor_id for t in sch.tensors.values() if t.resident]
    assert "embd" in resident and sum(sch.tensors[t].size for t in resident if t != "embd") <= 300


def test_gguf_read_parallel_matches_memory_map(tmp_path):
    from air_rs.gguf import GGMLType, read_gguf
    from air_rs.models.config import tiny_llama
    from air_rs.models.random_init import write_random_gguf
    p = tmp_path / "m.gguf"
    write_random_gguf(str(p), tiny_llama(), GGMLType.Q8_0, seed=0)
    g = read_gguf(str(p))
    bufs = g.read_parallel(workers=4, pin=False)
    assert set(bufs) == set(g.tensors)
    for n in g.tensors:
        assert torch.equal(bufs[n], g.raw(n)), n


def test_native_vram_arena_and_ram_pool():
    """Native STRIX budget arena (reference src/strix/arena.rs) and RAM pool (ram_pool.rs)."""
    from air_rs.stream.strix import ram_pool, vram_arena
    a = vram_arena(1 << 20, 4096)
    assert a.usable == (1 << 20) - 4096 and a.available == a.usable
    x = a.allocate(1000, 256)
    y = a.allocate(5000, 4096)
    assert x.offset == 0 and y.offset % 4096 == 0 and y.offset >= 1000
    assert a.used == 6000 and a.fragment_count() == 2          # the alignment gap stays free
    a.free(x)
    a.free(y)
    assert a.used == 0 and a.fragment_count() == 1 and a.largest_free() == a.usable
    with pytest.raises(ValueError):
        a.free(y)                                                 # double free is caught
    assert a.allocate(a.usable + 1, 1) is None                    # out of budget
    a.register_flight_slots(3, 65536, 4096)
    order = [a.next_flight_slot().index for _ in range(5)]
    assert order == [0, 1, 2, 0, 1]
    s = a.flight_slots[2]
    s.timeline_value = 7
    assert a.flight_slots[2].timeline_value == 7
    p = ram_pool(1 << 16)
    b = p.acquire(5000)
    assert len(b) == 5000 and b.capacity == 8192
    mv = memoryview(b)
    mv[:4] = b"abcd"
    addr = b.address
    del mv
    assert p.release(b) and p.pool_bytes == 8192
    c = p.acquire(6000)                                           # same class: recycled storage
    assert c.address == addr and p.recycled_count == 1 and p.pool_bytes == 0
    big = p.acquire(1 << 17)
    assert not p.release(big)                                     # above the cap: freed


def test_cold_boot_plan_phases():
    """Cold boot order (reference src/strix/cold_boot.rs:76-170)."""
    from air_rs.stream.strix import TensorClass, plan_cold_boot
    ts = [("output.weight", TensorClass.A, None, 100), ("blk.3.w", TensorClass.B, 3, 10),
          ("blk.0.w", TensorClass.B, 0, 10), ("blk.1.w", TensorClass.B, 1, 10),
          ("draft.w", TensorClass.C, None, 7), ("expert.9", TensorClass.D, 5, 3)]
    plan = plan_cold_boot(ts, prefetch_window=2)
    assert [(s.name, s.phase) for s in plan.steps] == [
        ("output.weight", 1), ("blk.0.w", 2), ("blk.1.w", 2), ("blk.3.w", 3), ("draft.w", 4)]
    assert plan.skipped == 1 and plan.critical_path_bytes == 120 and plan.total_transfer_bytes == 130
    assert abs(plan.estimate_ttft_seconds(120 / 2**20) - 1.0) < 1e-9
