"""Memory pressure levels / actions (reference src/strix/vram_pressure.rs tests) and the KV
pool controller acting on an engine."""
import pytest

from air_rs.runtime.pressure import (KvPressureController, PressureLevel, VramPressureManager,
                                     kv_cache_budget)


def test_levels_and_actions():
    m = VramPressureManager(8 << 30, 512 << 20, 3)
    assert m.budget == (8 << 30) - (512 << 20)
    b = m.budget
    assert m.evaluate(b // 2) == PressureLevel.GREEN
    assert m.evaluate(int(b * 0.62)) == PressureLevel.YELLOW
    assert m.evaluate(int(b * 0.80)) == PressureLevel.ORANGE
    assert m.evaluate(int(b * 0.90)) == PressureLevel.RED
    assert m.evaluate(b) == PressureLevel.CRITICAL
    assert VramPressureManager(0).evaluate(0) == PressureLevel.CRITICAL
    assert m.recommended_actions(PressureLevel.YELLOW)[0].value == 1
    assert [a.kind for a in m.recommended_actions(PressureLevel.RED)] == ["evict_class", "suspend_prefetch", "compress_kv"]
    assert m.recommended_flight_slot_size(PressureLevel.CRITICAL) == 64 << 20
    assert kv_cache_budget(4096, 8, 128, 32) == 2 * 4096 * 8 * 128 * 32 * 2
    assert str(PressureLevel.ORANGE) == "Orange (75-85%)"


class _Alloc:
    def __init__(self, total, used):
        self.t, self.u = total, used

    @property
    def total_blocks(self):
        return self.t

    def num_used_blocks(self):
        return self.u


class _Cache:
    def __init__(self, n, alloc):
        self.n, self.alloc = n, alloc

    def size(self):
        return self.n

    def evict_until(self, k):
        k = min(k, self.n)
        self.n -= k
        self.alloc.u -= k
        return k


class _Seqs:
    def __init__(self, alloc):
        self.allocator = alloc


class _Eng:
    def __init__(self, total, used, cached):
        a = _Alloc(total, used)
        self.seqs = _Seqs(a)
        self.prefix_cache = _Cache(cached, a)
        self.swap = object()
        self.running = [1, 2, 3]
        self.admit_paused = False
        self.preempts = 0

    def preempt_latest(self):
        self.preempts += 1
        self.running.pop()
        return True


@pytest.mark.parametrize("used,level,paused,evicted,preempt", [
    (50, PressureLevel.GREEN, False, 0, 0),
    (80, PressureLevel.ORANGE, False, 10, 0),
    (90, PressureLevel.RED, True, 20, 0),
    (97, PressureLevel.CRITICAL, True, 30, 1),
])
def test_controller_actions(used, level, paused, evicted, preempt):
    e = _Eng(100, used, 30)
    c = KvPressureController(e)
    assert c.tick() == level
    assert e.admit_paused == paused and c.evicted_blocks == evicted and e.preempts == preempt


def test_controller_with_native_allocator():
    from air_rs import _host
    seqs = _host.SequenceManager(20, 16)
    e = _Eng(1, 0, 0)
    e.seqs, e.prefix_cache = seqs, None
    c = KvPressureController(e)
    assert c.mgr.budget == 20 and c.tick() == PressureLevel.GREEN
    s = seqs.create_sequence()
    seqs.append(s, 16 * 19)
    assert c.tick() == PressureLevel.CRITICAL and e.admit_paused and e.preempts == 1
