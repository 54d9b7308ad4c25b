"""End-to-end engine on the GPU vs the reference-numerics CPU oracle (teacher forcing)."""
import pytest
import torch

from air_rs.gguf import GGMLType
from air_rs.models.config import tiny_llama
from air_rs.models.random_init import random_tensors
from air_rs.models.reference import OracleModel, apply_repetition_penalty
from air_rs.runtime.builder import build_runner
from air_rs.runtime.engine import Engine, SamplingParams

pytestmark = pytest.mark.gpu


def _models(qt, max_batch=16):
    cfg = tiny_llama()
    recs = list(random_tensors(cfg, qt, seed=0, device="cpu"))
    oracle = OracleModel(cfg, {n: (r, q, s) for n, r, q, s in recs})
    runner = build_runner(cfg, iter(recs), device="cuda", max_batch=max_batch, max_model_len=512,
                          num_blocks=512)
    return cfg, oracle, runner


def _check_near_argmax(oracle, prompt, toks, penalty=1.1, tol=0.15):
    """Teacher-force the GPU's tokens through the oracle; each must be near its argmax."""
    oracle.reset()
    seq = list(prompt)
    logits = oracle.forward(seq, 0)
    worst = 0.0
    for t in toks:
        lg = apply_repetition_penalty(logits, seq, penalty)
        gap = float(lg.max() - lg[t])
        worst = max(worst, gap)
        seq.append(t)
        logits = oracle.forward([t], len(seq) - 1)
    spread = float(lg.max() - lg.min())
    assert worst <= tol * spread, (worst, spread)
    return worst


@pytest.mark.parametrize("qt", [GGMLType.Q8_0, GGMLType.Q4_K])
def test_engine_gemv_path_matches_oracle(qt):
    cfg, oracle, runner = _models(qt)
    eng = Engine(cfg, runner, max_batch=8)
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, cfg.vocab_size, (32,), generator=g).tolist()
    out = eng.generate_ids([prompt], SamplingParams(max_tokens=24, temperature=0.0, ignore_eos=True))[0]
    assert len(out) == 24
    _check_near_argmax(oracle, [cfg.bos_token_id] + prompt, out)


def test_engine_batched_gemm_path_and_pipelining():
    cfg, oracle, runner = _models(GGMLType.Q4_K, max_batch=16)
    eng = Engine(cfg, runner, max_batch=16)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, cfg.vocab_size, (int(n),), generator=g).tolist()
               for n in torch.randint(5, 60, (12,), generator=g)]
    params = SamplingParams(max_tokens=20, temperature=0.0, ignore_eos=True)
    outs = eng.generate_ids(prompts, params, pipelined=True)
    assert all(len(o) == 20 for o in outs)
    for p, o in zip(prompts[:3], outs[:3]):
        _check_near_argmax(oracle, [cfg.bos_token_id] + p, o)
    # all KV blocks returned to the pool
    assert eng.seqs.allocator.num_used_blocks() == 0


def test_sampling_is_reproducible():
    cfg, oracle, runner = _models(GGMLType.Q8_0)
    g = torch.Generator().manual_seed(2)
    prompt = torch.randint(0, cfg.vocab_size, (16,), generator=g).tolist()
    params = SamplingParams(max_tokens=16, temperature=0.8, top_k=40, top_p=0.9, ignore_eos=True)
    a = Engine(cfg, runner, max_batch=8).generate_ids([prompt], params)[0]
    runner.step_ctr.zero_()
    b = Engine(cfg, runner, max_batch=8).generate_ids([prompt], params)[0]
    assert a == b
