"""Ghost drafting policy (reference src/ghost_drafting.rs tests): model selection,
feasibility, acceptance tracking with adaptive draft length, checkpoint-tree rollback."""
import pytest

from air_rs.spec.ghost import (AcceptanceTracker, GhostModel, GhostPlatformProfile, GhostSession,
                               SpeculativeCheckpointTree, check_feasibility, feasibility_matrix,
                               select_ghost_model)


def test_select_and_sizes():
    assert select_ghost_model(8000) == GhostModel.LLAMA32_3B
    assert select_ghost_model(2500) == GhostModel.LLAMA32_1B
    assert select_ghost_model(1000) is None
    assert GhostModel.LLAMA32_1B.size_mb == 700.0 and "1.9 GB" in str(GhostModel.LLAMA32_3B)


def test_feasibility():
    p = GhostPlatformProfile.nvidia_gpu()
    assert check_feasibility(1062.0, p, False).feasible
    assert not check_feasibility(50.0, p, False).feasible
    r = check_feasibility(1062.0, p, True)
    assert not r.applicable and not r.feasible
    m = feasibility_matrix(p, 85.0)
    assert m[0].storage_name == "USB 3.0 HDD" and m[0].feasible and not m[-1].feasible


def test_tracker_ema_and_adaptive_k():
    t = AcceptanceTracker()
    assert t.acceptance_rate() == 0.75
    for _ in range(10):
        t.report_batch(4, 4)
    assert t.ema_rate > 0.85 and t.suggest_k() == 6 and t.acceptance_rate() == 1.0
    t2 = AcceptanceTracker()
    for _ in range(5):
        t2.report_batch(4, 0)
    assert t2.should_disable() and t2.suggest_k() == 1
    t3 = AcceptanceTracker(draft_k=4, ema_rate=0.5)
    assert t3.suggest_k() == 3
    t3.report_batch(4, 9)                 # accepted is clamped to drafted
    assert t3.total_accepted == 4
    assert abs(AcceptanceTracker().net_ghost_contribution_ms(70.0) - 157.5) < 1e-9


def test_session_auto_disables():
    s = GhostSession.create(8000, GhostPlatformProfile.nvidia_gpu(), 1062.0)
    assert s.active and s.perceived_ttft_ms() == 85.0 and s.ttft_speedup() > 10
    for _ in range(5):
        s.report_verification(4, 0)
    assert not s.active and s.ttft_speedup() == 1.0 and s.rho_contribution(70) == 0.0


def test_checkpoint_tree_rollback():
    c = SpeculativeCheckpointTree(3)
    for off, tok in [(0, 10), (1, 11), (2, 12)]:
        c.push_diff(off, tok)
    assert c.tokens_after([1, 2, 3, 4, 5]) == [1, 2, 3, 10, 11, 12]
    assert c.rollback(1) == 4 and c.tokens_after([1, 2, 3]) == [1, 2, 3, 10]


@pytest.mark.gpu
def test_adaptive_draft_depth_keeps_greedy_output():
    from air_rs.runtime.builder import random_engine
    from air_rs.spec.speculative import SpeculativeDecoder
    from test_spec import _greedy_margin
    tgt = random_engine("tiny", seed=1, device="cuda:0", max_batch=8, max_model_len=512)
    dft = random_engine("tiny", seed=1, device="cuda:0", max_batch=8, max_model_len=512)
    sd = SpeculativeDecoder(tgt, dft, k=2, tau=0.0, eos_id=-1, adaptive=True, k_max=6)
    prompt = [3, 17, 29, 41, 5]
    outs, stats = sd.generate_batch([prompt], max_tokens=32)
    gap, spread = _greedy_margin(tgt, prompt, outs[0])
    assert (gap <= 0.05 * spread).all()
    assert sd.k > 2 and sd.tracker.batch_count() > 0     # identical draft: depth grows
