"""Evaluation harness (reference src/eval.rs tests) on the CPU oracle engine."""
import math

import pytest
import torch

from air_rs.eval import (Arc, BenchmarkResult, BenchmarkRunner, EngineScorer, HellaSwag, Mmlu,
                         MultipleChoiceQuestion, RegressionError, TokenPerplexity, greedy_match_rate)


def test_result_tolerance_rules():
    assert BenchmarkResult("a", 0.70, "accuracy", 10).within_tolerance(0.71, 0.02)
    assert not BenchmarkResult("a", 0.60, "accuracy", 10).within_tolerance(0.71, 0.02)
    assert BenchmarkResult("p", 10.1, "perplexity", 10).within_tolerance(10.0, 0.02)
    assert not BenchmarkResult("p", 11.0, "perplexity", 10).within_tolerance(10.0, 0.02)


def test_multiple_choice_acc_norm():
    q = MultipleChoiceQuestion("ctx", ["a b c d", "x"], 0)
    # per-token normalisation: -4/4 = -1 beats -2/1
    assert q.pick(lambda c, s: -4.0 if s == "a b c d" else -2.0) == 0
    bench = HellaSwag([q, MultipleChoiceQuestion("ctx", ["y", "z"], 1)], 0)
    r = bench.evaluate(lambda c, s: {"a b c d": -4.0, "x": -2.0, "y": -1.0, "z": -3.0}[s])
    assert r.score == 0.5 and r.n_examples == 2 and r.name == "hellaswag"


def test_jsonl_loaders(tmp_path):
    p = tmp_path / "hs.jsonl"
    p.write_text('{"ctx": "A man", "endings": ["runs", "flies"], "label": 0}\n')
    assert HellaSwag.from_jsonl(str(p)).questions[0].choices == ["runs", "flies"]
    p = tmp_path / "arc.jsonl"
    p.write_text('{"question": "Q?", "choices": {"text": ["x", "y"], "label": ["A", "B"]}, "answerKey": "B"}\n')
    assert Arc.from_jsonl(str(p)).questions[0].correct_idx == 1
    d = tmp_path / "mmlu"
    d.mkdir()
    (d / "algebra.jsonl").write_text('{"question": "1+1", "choices": ["1", "2"], "answer": 1}\n')
    m = Mmlu.from_dir(str(d))
    assert m.questions[0].subject == "algebra"


def test_rolling_perplexity_scores_each_token_once():
    ids = list(range(10))
    seen = []

    def lp(window):
        seen.append(list(window))
        return [math.log(0.5)] * (len(window) - 1)
    r = TokenPerplexity(ids, stride=3, max_length=5).evaluate_tokens(lp)
    assert r.n_examples == 9 and abs(r.score - 2.0) < 1e-9


@pytest.fixture(scope="module")
def cpu_engine(tmp_path_factory):
    from air_rs.gguf import GGMLType
    from air_rs.models.config import tiny_llama
    from air_rs.models.random_init import write_random_gguf
    from air_rs.runtime.builder import engine_from_gguf
    path = tmp_path_factory.mktemp("m") / "tiny.gguf"
    write_random_gguf(str(path), tiny_llama(), GGMLType.Q8_0, seed=0)
    return engine_from_gguf(str(path), device="cpu")


def test_engine_scorer_and_gate_on_oracle(cpu_engine):
    eng = cpu_engine
    lp = eng.token_logprobs([5, 6, 7])
    assert len(lp) == 3 and all(v < 0 for v in lp)
    scorer = EngineScorer(eng)
    runner = BenchmarkRunner(tolerance=0.0)
    runner.add_benchmark(TokenPerplexity(list(range(3, 40)), stride=16, max_length=24))
    runner.add_benchmark(Mmlu.stub())
    res = runner.run(scorer)
    ppl = res[0].score
    assert 1.0 < ppl < 2 * eng.cfg.vocab_size
    runner.set_baseline("wikitext103_ppl", ppl * 0.5)
    with pytest.raises(RegressionError):
        runner.run(scorer)
    assert greedy_match_rate(eng, eng.oracle, [[9, 10, 11]], 3) == 1.0


@pytest.mark.gpu
def test_gpu_token_logprobs_match_oracle():
    from air_rs.gguf import GGMLType
    from air_rs.models.config import tiny_llama
    from air_rs.models.random_init import random_tensors
    from air_rs.models.reference import OracleModel
    from air_rs.runtime.builder import build_runner
    from air_rs.runtime.engine import Engine
    cfg = tiny_llama()
    recs = list(random_tensors(cfg, GGMLType.Q8_0, seed=0, device="cpu"))
    oracle = OracleModel(cfg, {n: (r, q, s) for n, r, q, s in recs})
    eng = Engine(cfg, build_runner(cfg, iter(recs), device="cuda", max_batch=8, max_model_len=256, num_blocks=64))
    ref = Engine(cfg, None, oracle=oracle)
    ids = torch.randint(0, cfg.vocab_size, (40,), generator=torch.Generator().manual_seed(0)).tolist()
    a, b = torch.tensor(eng.token_logprobs(ids)), torch.tensor(ref.token_logprobs(ids))
    assert a.shape == b.shape == (40,)
    torch.testing.assert_close(a, b, rtol=0, atol=0.05)
    assert eng.seqs.allocator.num_used_blocks() == 0
