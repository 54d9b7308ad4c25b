"""Speculative decoding: EAGLE-2 tree construction / acceptance on CPU, the tree-verify
decoder on the GPU (reference tests in ``src/eagle2.rs`` and ``src/speculative.rs``)."""
import math

import pytest
import torch

from air_rs.spec.eagle2 import (DRAFT_TOP_K, EXPAND_THRESHOLD, MAX_TREE_DEPTH, DraftNode, DraftTree, Eagle2Builder,
                                accept_sample, greedy_accept)


class _PeakedDraft:
    """Next token = (last + 1) % V with probability 0.7, the rest spread over 3 others."""

    def __init__(self, V=16):
        self.V = V

    def next_logits(self, ctx):
        p = torch.full((self.V,), 1e-6)
        t = ctx[-1]
        p[(t + 1) % self.V] = 0.7
        p[(t + 2) % self.V] = 0.2
        p[(t + 3) % self.V] = 0.06
        p[(t + 4) % self.V] = 0.04
        return p.log()


def test_constants_match_reference():
    assert (MAX_TREE_DEPTH, EXPAND_THRESHOLD, DRAFT_TOP_K) == (6, 0.05, 4)


def test_builder_expands_above_threshold_only():
    tree = Eagle2Builder(_PeakedDraft(), max_depth=3).build([5])
    assert tree.nodes[0].parent_idx is None and tree.nodes[0].token_id == 6
    roots = tree.children(None)
    assert [tree.nodes[i].token_id for i in roots] == [6, 7, 8, 9]
    # the 0.04 child is below tau: it gets no children; the others do
    assert tree.children(roots[3]) == []
    assert all(len(tree.children(r)) == 4 for r in roots[:3])
    assert max(n.depth for n in tree.nodes) == 2
    for n in tree.nodes:
        if n.parent_idx is not None:
            assert n.depth == tree.nodes[n.parent_idx].depth + 1
            assert abs(n.cum_prob - tree.nodes[n.parent_idx].cum_prob * n.draft_prob) < 1e-6


def test_max_nodes_cap():
    tree = Eagle2Builder(_PeakedDraft(), tau=0.0, max_depth=6, max_nodes=20).build([0])
    assert len(tree) == 20


def test_tree_mask_and_bits():
    t = DraftTree(1, [DraftNode(1, 1, 0, None), DraftNode(2, .5, 1, 0), DraftNode(3, .4, 1, 0),
                      DraftNode(4, .3, 2, 1)])
    m = t.to_mask()
    assert m.tolist() == [[1, 0, 0, 0], [1, 1, 0, 0], [1, 0, 1, 0], [1, 1, 0, 1]]
    assert t.ancestor_bits() == [0b1, 0b11, 0b101, 0b1011]
    assert t.ancestor_bits(2)[3] == 0b1011 << 2
    assert sorted(t.all_paths()) == [[0, 1, 3], [0, 2]]
    assert t.flatten() == [1, 2, 3, 4]


def test_greedy_accept_follows_matching_children():
    t = DraftTree(1, [DraftNode(1, 1, 0, None), DraftNode(2, .5, 1, 0), DraftNode(3, .4, 1, 0),
                      DraftNode(4, .3, 2, 2)])
    # target after root -> 3 (node 2), after node 2 -> 4 (node 3), after node 3 -> 9 (bonus)
    path, bonus = greedy_accept(t, [3, 0, 4, 9])
    assert path == [0, 2, 3] and bonus == 9
    path, bonus = greedy_accept(t, [7, 0, 0, 0])
    assert path == [0] and bonus == 7


def test_accept_sample_identical_distributions_accepts_all():
    p = torch.tensor([0.1, 0.6, 0.3])
    r = accept_sample([1, 2], [p, p], [p, p], rng=lambda: 0.999)
    assert r.n_accepted == 2 and r.bonus_token == -1


def test_accept_sample_residual_is_exact():
    """P(out = x) over accept/reject must equal the target p(x) (one position)."""
    p = torch.tensor([0.5, 0.3, 0.2])
    q = torch.tensor([0.2, 0.7, 0.1])
    gen = torch.Generator().manual_seed(0)
    counts = torch.zeros(3)
    n = 40000
    for _ in range(n):
        x = int(torch.multinomial(q, 1, generator=gen))
        r = accept_sample([x], [p], [q], rng=lambda: torch.rand((), generator=gen).item())
        counts[x if r.n_accepted == 1 else r.bonus_token] += 1
    assert torch.allclose(counts / n, p, atol=0.015)


# ---------------------------------------------------------------------------------------- GPU
def _greedy_margin(eng, prompt, out):
    """Per emitted token: max logit minus the emitted token's logit under one full forward."""
    rn = eng.runner
    dev = rn.device
    seq = [eng.cfg.bos_token_id] + prompt + out
    s = eng.seqs.create_sequence()
    try:
        slots = eng.seqs.append(s, len(seq))
        tab = torch.full((1, rn.max_blocks), -1, dtype=torch.int32)
        eng.seqs.fill_table([s], tab)
        T = len(seq)
        lg = rn.prefill(torch.tensor(seq, dtype=torch.int32, device=dev),
                        torch.arange(T, dtype=torch.int32, device=dev),
                        torch.tensor(slots, dtype=torch.int64, device=dev),
                        torch.zeros(T, dtype=torch.int32, device=dev), tab.to(dev),
                        torch.arange(T, dtype=torch.int64, device=dev), None, None, None, None, None,
                        return_logits=True).float().cpu()
    finally:
        eng.seqs.free_sequence(s)
    n0 = 1 + len(prompt) - 1
    rows = lg[n0:n0 + len(out)]
    picked = rows.gather(1, torch.tensor(out)[:, None]).squeeze(1)
    return rows.max(1).values - picked, rows.std(1)


@pytest.mark.gpu
@pytest.mark.parametrize("same_draft", [True, False])
def test_speculative_greedy_matches_target(same_draft):
    from air_rs.runtime.builder import random_engine
    from air_rs.spec.speculative import SpeculativeDecoder
    tgt = random_engine("tiny", seed=1, device="cuda:0", max_batch=8, max_model_len=512)
    dft = random_engine("tiny", seed=1 if same_draft else 2, device="cuda:0", max_batch=8, max_model_len=512)
    sd = SpeculativeDecoder(tgt, dft, k=3, tau=0.0, max_nodes=32, eos_id=-1)
    used0 = [e.seqs.allocator.num_used_blocks() for e in (tgt, dft)]
    prompts = [[3, 17, 29, 41, 5], [100, 7, 7, 9]]
    outs, stats = sd.generate_batch(prompts, max_tokens=24)
    assert all(len(o) == 24 for o in outs)
    for p, o in zip(prompts, outs):
        gap, spread = _greedy_margin(tgt, p, o)
        # every emitted token is the target's argmax up to bf16 noise between the two forwards
        assert (gap <= 0.05 * spread).all(), (gap, spread)
    if same_draft:
        assert stats.acceptance_rate > 0 and stats.tokens_per_round > 2.5, str(stats)
    # all KV blocks returned
    assert [e.seqs.allocator.num_used_blocks() for e in (tgt, dft)] == used0
    tgt.runner.check_errors()


@pytest.mark.gpu
def test_speculative_sampling_runs():
    from air_rs.runtime.builder import random_engine
    from air_rs.spec.speculative import SpeculativeDecoder
    tgt = random_engine("tiny", seed=1, device="cuda:0", max_batch=8, max_model_len=512)
    sd = SpeculativeDecoder(tgt, tgt, k=2, eos_id=-1)
    out, stats = sd.generate([1, 2, 3], max_tokens=16, temperature=0.8, seed=3)
    assert len(out) == 16 and stats.rounds >= 1


def test_jsd_properties():
    from air_rs.spec.medusa import jsd
    p = torch.tensor([0.5, 0.5, 0.0])
    q = torch.tensor([0.0, 0.5, 0.5])
    assert jsd([p, p, p]) == 0.0
    assert 0 < jsd([p, q]) <= math.log(2) + 1e-6


@pytest.mark.gpu
def test_medusa_and_council_verify_with_target():
    from air_rs.gguf import GGMLType
    from air_rs.models.config import tiny_llama
    from air_rs.models.random_init import random_tensors
    from air_rs.models.reference import OracleModel
    from air_rs.runtime.builder import build_runner
    from air_rs.runtime.engine import Engine
    from air_rs.spec.medusa import CouncilDecoder, MedusaDecoder, MedusaHeads
    from test_engine_gpu import _check_near_argmax
    cfg = tiny_llama()
    recs = list(random_tensors(cfg, GGMLType.Q8_0, seed=0, device="cpu"))
    oracle = OracleModel(cfg, {n: (r, q, s) for n, r, q, s in recs})
    mk = lambda: Engine(cfg, build_runner(cfg, iter(recs), device="cuda", max_batch=8, max_model_len=512,
                                          num_blocks=128))
    tgt = mk()
    prompt = [3, 17, 29, 41, 5, 77]
    md = MedusaDecoder(tgt, MedusaHeads(cfg.hidden_dim, 3, "cuda"), top_c=2, eos_id=-1)
    out, st = md.generate(prompt, 16)
    assert len(out) == 16 and st.rounds >= 1 and st.drafted > 0
    _check_near_argmax(oracle, [cfg.bos_token_id] + prompt, out, penalty=1.0)
    used = tgt.seqs.allocator.num_used_blocks()
    cd = CouncilDecoder(tgt, [mk(), mk()], epsilon=0.05, k=3, eos_id=-1)
    out, st = cd.generate(prompt, 16)
    assert len(out) == 16
    _check_near_argmax(oracle, [cfg.bos_token_id] + prompt, out, penalty=1.0)
    # identical voters always agree, and they are the target itself: drafts are accepted
    assert max(cd.jsd_history) < 1e-6 and st.tokens_per_round > 2.0, str(st)
    assert tgt.seqs.allocator.num_used_blocks() == used
