"""Evaluation harness (reference ``src/eval.rs``): multiple-choice benchmarks (HellaSwag, ARC,
MMLU) scored by length-normalised log-likelihood (``acc_norm``), perplexity over a token
stream with a rolling window, and a regression gate against baselines.

The reference's perplexity benchmark scores placeholder strings; here every number comes
from the model: ``EngineScorer`` turns ``Engine.token_logprobs`` (one forward over the whole
sequence on the GPU) into the ``score(context, continuation)`` callback the benchmarks use.
``greedy_match_rate`` is the numerics gate against the reference-numerics CPU oracle.
"""
from __future__ import annotations

import json
import math
import os
from dataclasses import dataclass, field
from typing import Callable, Protocol

ScoreFn = Callable[[str, str], float]


@dataclass
class BenchmarkResult:
    name: str
    score: float
    metric: str
    n_examples: int
    breakdown: list[tuple[str, float]] = field(default_factory=list)

    def within_tolerance(self, baseline: float, tolerance: float) -> bool:
        """Accuracy may drop by at most ``tolerance``; perplexity may rise by that fraction."""
        if self.metric == "perplexity":
            return self.score <= baseline * (1.0 + tolerance)
        return self.score >= baseline - tolerance


class Benchmark(Protocol):
    name: str
    n_shot: int

    def evaluate(self, score_fn: ScoreFn) -> BenchmarkResult: ...


@dataclass
class MultipleChoiceQuestion:
    context: str
    choices: list[str]
    correct_idx: int
    subject: str = ""

    def pick(self, score_fn: ScoreFn) -> int:
        """Index of the choice with the highest log-likelihood per whitespace token."""
        best, best_v = 0, -math.inf
        for i, c in enumerate(self.choices):
            v = score_fn(self.context, c) / max(1, len(c.split()))
            if v > best_v:
                best, best_v = i, v
        return best

    def score(self, score_fn: ScoreFn) -> bool:
        return self.pick(score_fn) == self.correct_idx


def _load_jsonl(path: str, ctx_key: str, choices_key: str, label_key: str) -> list[MultipleChoiceQuestion]:
    out = []
    with open(path) as f:
        for line in f:
            if not line.strip():
                continue
            d = json.loads(line)
            ch = d[choices_key]
            if isinstance(ch, dict):                     # ARC: {"text": [...], "label": [...]}
                labels, ch = ch.get("label", []), ch["text"]
                lab = d[label_key]
                idx = labels.index(lab) if lab in labels else int(lab)
            else:
                idx = int(d[label_key])
            out.append(MultipleChoiceQuestion(d[ctx_key], list(ch), idx, d.get("subject", "")))
    return out


class MultipleChoiceBenchmark:
    metric = "accuracy"

    def __init__(self, name: str, questions: list[MultipleChoiceQuestion], n_shot: int = 0):
        self.name, self.questions, self.n_shot = name, questions, n_shot

    def evaluate(self, score_fn: ScoreFn) -> BenchmarkResult:
        by_subj: dict[str, list[bool]] = {}
        for q in self.questions:
            by_subj.setdefault(q.subject, []).append(q.score(score_fn))
        flat = [x for v in by_subj.values() for x in v]
        acc = sum(flat) / len(flat) if flat else 0.0
        res = BenchmarkResult(self.name, acc, self.metric, len(flat))
        if len(by_subj) > 1:
            res.breakdown = [(k, sum(v) / len(v)) for k, v in sorted(by_subj.items())]
        return res


class HellaSwag(MultipleChoiceBenchmark):
    def __init__(self, questions, n_shot: int = 10):
        super().__init__("hellaswag", questions, n_shot)

    @classmethod
    def from_jsonl(cls, path: str, n_shot: int = 10):
        return cls(_load_jsonl(path, "ctx", "endings", "label"), n_shot)

    @classmethod
    def stub(cls):
        return cls([MultipleChoiceQuestion("The sun rises in the", ["east", "west", "sea", "night"], 0)], 0)


class Arc(MultipleChoiceBenchmark):
    def __init__(self, questions, split: str = "easy", n_shot: int = 25):
        super().__init__(f"arc_{split}", questions, n_shot)

    @classmethod
    def from_jsonl(cls, path: str, split: str = "easy"):
        return cls(_load_jsonl(path, "question", "choices", "answerKey"), split)

    @classmethod
    def stub(cls, split: str = "easy"):
        return cls([MultipleChoiceQuestion("Water freezes at", ["0 C", "50 C", "100 C"], 0)], split, 0)


class Mmlu(MultipleChoiceBenchmark):
    def __init__(self, questions, n_shot: int = 5):
        super().__init__("mmlu", questions, n_shot)

    @classmethod
    def from_dir(cls, path: str, n_shot: int = 5):
        qs = []
        for fn in sorted(os.listdir(path)):
            if fn.endswith(".jsonl"):
                subj = fn[:-6]
                for q in _load_jsonl(os.path.join(path, fn), "question", "choices", "answer"):
                    q.subject = subj
                    qs.append(q)
        return cls(qs, n_shot)

    @classmethod
    def stub(cls):
        return cls([MultipleChoiceQuestion("2 + 2 =", ["3", "4", "5", "22"], 1, "math")], 0)


class TokenPerplexity:
    """Rolling-window perplexity over a token stream: each window of ``max_length`` tokens
    advances by ``stride``, and only the tokens new to a window are scored."""
    metric = "perplexity"

    def __init__(self, token_ids: list[int], stride: int = 512, max_length: int = 1024,
                 name: str = "wikitext103_ppl"):
        self.token_ids, self.stride, self.max_length, self.name, self.n_shot = token_ids, stride, max_length, name, 0

    def evaluate_tokens(self, logprob_fn: Callable[[list[int]], list[float]]) -> BenchmarkResult:
        ids = self.token_ids
        nll, n, prev_end = 0.0, 0, 0
        for begin in range(0, max(1, len(ids) - 1), self.stride):
            end = min(begin + self.max_length, len(ids))
            lp = logprob_fn(ids[begin:end])          # len = end - begin - 1 (token i | before i)
            new = end - max(prev_end, begin + 1)
            if new > 0:
                nll -= sum(lp[-new:])
                n += new
            prev_end = end
            if end == len(ids):
                break
        ppl = math.exp(nll / n) if n else float("inf")
        return BenchmarkResult(self.name, ppl, self.metric, n)

    def evaluate(self, score_fn: ScoreFn) -> BenchmarkResult:
        raise TypeError("TokenPerplexity needs a token log-prob function: use evaluate_tokens")


class BenchmarkRunner:
    def __init__(self, tolerance: float = 0.01):
        self.tolerance = tolerance
        self.benchmarks: list = []
        self.baselines: dict[str, float] = {}

    def add_benchmark(self, b):
        self.benchmarks.append(b)

    def set_baseline(self, name: str, score: float):
        self.baselines[name] = score

    def run(self, scorer: "EngineScorer") -> list[BenchmarkResult]:
        """Runs every benchmark; raises ``RegressionError`` listing the gates that failed."""
        results = []
        for b in self.benchmarks:
            if isinstance(b, TokenPerplexity):
                results.append(b.evaluate_tokens(scorer.token_logprobs))
            else:
                results.append(b.evaluate(scorer.score))
        bad = [f"{r.name}: score={r.score:.4f} baseline={self.baselines[r.name]:.4f} "
               f"tolerance={self.tolerance} metric={r.metric}"
               for r in results if r.name in self.baselines
               and not r.within_tolerance(self.baselines[r.name], self.tolerance)]
        if bad:
            raise RegressionError(bad, results)
        return results


class RegressionError(Exception):
    def __init__(self, regressions, results):
        super().__init__("; ".join(regressions))
        self.regressions, self.results = regressions, results


class EngineScorer:
    """Log-likelihood scoring through an ``air_rs.runtime.engine.Engine``."""

    def __init__(self, engine, tokenizer=None):
        self.engine = engine
        self.tok = tokenizer or engine.tokenizer

    def token_logprobs(self, ids: list[int]) -> list[float]:
        return self.engine.token_logprobs(ids, add_bos=False)

    def score(self, context: str, continuation: str) -> float:
        """log p(continuation | context), summed over the continuation's tokens."""
        c = self.tok.encode(context)
        full = self.tok.encode(context + continuation)
        k = len(full) - len(c)
        if k <= 0:
            return 0.0
        lp = self.engine.token_logprobs(full)        # BOS prepended: one entry per token
        return float(sum(lp[-k:]))


def greedy_match_rate(engine, oracle, prompts: list[list[int]], n_tokens: int) -> float:
    """Fraction of greedy tokens the engine shares with the reference-numerics oracle
    (teacher-forced: the oracle predicts each next token from the engine's prefix)."""
    import torch
    from .runtime.engine import SamplingParams
    outs = engine.generate_ids(prompts, SamplingParams(max_tokens=n_tokens, temperature=0.0,
                                                       repetition_penalty=1.0, ignore_eos=True))
    same = total = 0
    bos = [engine.cfg.bos_token_id] if engine.add_bos else []
    for p, o in zip(prompts, outs):
        oracle.reset()
        seq = bos + list(p)
        logits = oracle.forward(seq, 0)
        for t in o:
            same += int(int(torch.argmax(logits)) == t)
            total += 1
            seq.append(t)
            logits = oracle.forward([t], len(seq) - 1)
    oracle.reset()
    return same / total if total else 1.0
