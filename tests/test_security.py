"""Memory-safety helpers (reference src/strix/security.rs tests)."""
import threading

import pytest
import torch

from air_rs.utils.security import (BoundsCheckedRegion, BoundsError, OwnerToken, SecureAllocator,
                                   SecurityAuditLog, ShardedRwLock, zero_kv_blocks)


def test_audit_ring_and_hmac_chain():
    log = SecurityAuditLog(capacity=16)
    for i in range(20):
        log.log("allocated", handle=i)
    assert len(log) == 16 and log.total_logged == 20
    evs = log.ordered()
    assert [e.detail["handle"] for e in evs] == list(range(4, 20))
    assert log.verify()
    evs[5].detail["handle"] = 999          # tamper with one entry
    assert not log.verify(evs)


def test_bounds_and_owner():
    log = SecurityAuditLog()
    buf = torch.arange(100)
    a, b = OwnerToken(1), OwnerToken(2)
    r = BoundsCheckedRegion(buf, 10, 20, a, log)
    assert r.view(0, 5, a).tolist() == [10, 11, 12, 13, 14]
    with pytest.raises(BoundsError):
        r.view(18, 5, a)
    with pytest.raises(BoundsError):
        r.view(0, 1, b)
    assert [e.kind for e in log.ordered()] == ["bounds_violation", "owner_violation"]
    with pytest.raises(BoundsError):
        BoundsCheckedRegion(buf, 90, 20, a)


def test_secure_allocator_zeroes():
    al = SecureAllocator()
    o = OwnerToken(7)
    h, t = al.allocate((4,), torch.float32, o)
    t.fill_(3.0)
    with pytest.raises(BoundsError):
        al.secure_free(h, OwnerToken(8))
    al.secure_free(h, o)
    assert float(t.abs().sum()) == 0 and al.active_allocations() == 0
    assert al.log.ordered()[-1].kind == "zeroed_and_freed"


def test_sharded_lock_and_kv_zero():
    lk = ShardedRwLock(4)
    total = []

    def work(i):
        lk.read(i, lambda: total.append(i))
    ts = [threading.Thread(target=work, args=(i,)) for i in range(16)]
    [t.start() for t in ts]
    [t.join() for t in ts]
    assert sorted(total) == list(range(16)) and lk.write(lambda: 5) == 5
    kv = torch.ones(2, 6, 2, 3)
    zero_kv_blocks(kv, [1, 4])
    assert float(kv[:, [1, 4]].sum()) == 0 and float(kv[:, [0, 2, 3, 5]].sum()) == 2 * 4 * 6


@pytest.mark.gpu
def test_engine_secure_kv_zeroes_freed_blocks():
    from air_rs.runtime.builder import random_engine
    from air_rs.runtime.engine import SamplingParams
    eng = random_engine("tiny", max_batch=4, max_model_len=256, num_blocks=64, secure_kv=True)
    rid = eng.add_request(list(range(3, 40)), SamplingParams(max_tokens=4, temperature=0.0, ignore_eos=True))
    eng.step()
    r = next(x for x in eng.running if x.rid == rid)
    blocks = list(eng.seqs.block_table(r.seq))
    assert float(eng.runner.kv[:, blocks].abs().sum()) > 0
    while eng.has_unfinished():
        eng.step()
    torch.cuda.synchronize()
    assert float(eng.runner.kv[:, blocks].abs().sum()) == 0
