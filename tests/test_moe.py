"""Mixture-of-experts: routing (reference src/moe.rs tests) on CPU, the device routing
kernel against a PyTorch restatement, and a tiny Mixtral-style model on the GPU against the
reference-numerics oracle."""
import pytest
import torch

from air_rs.gguf import GGMLType
from air_rs.models.config import tiny_moe
from air_rs.models.random_init import random_tensors
from air_rs.models.reference import OracleModel, compute_routing, greedy_generate


def test_compute_routing_top2_normalised():
    ids, w = compute_routing(torch.tensor([0.1, 2.0, -1.0, 1.5]), 2)
    assert ids == [1, 3]
    assert abs(float(w.sum()) - 1.0) < 1e-6 and float(w[0]) > float(w[1])
    ids, w = compute_routing(torch.tensor([1.0, 1.0, 1.0, 1.0]), 2, normalize=False)
    assert ids == [0, 1] and torch.allclose(w, torch.tensor([0.25, 0.25]))


def test_oracle_moe_forward_runs_and_routes():
    cfg = tiny_moe()
    recs = list(random_tensors(cfg, GGMLType.Q8_0, seed=0, device="cpu"))
    oracle = OracleModel(cfg, {n: (r, q, s) for n, r, q, s in recs})
    out = greedy_generate(oracle, [5, 6, 7, 8], 4, cfg.bos_token_id)
    assert len(out) == 4 and all(0 <= t < cfg.vocab_size for t in out)


@pytest.mark.gpu
def test_moe_route_kernel_matches_torch():
    from air_rs import ops
    ext = ops.require_ext()
    g = torch.Generator().manual_seed(0)
    T, H, E, k = 37, 512, 8, 2
    x = torch.randn(T, H, generator=g)
    router = torch.randn(E, H, generator=g) * 0.05
    cw = torch.zeros(T, E, device="cuda")
    ids = torch.zeros(T, k, dtype=torch.int32, device="cuda")
    wts = torch.zeros(T, k, device="cuda")
    ext.moe_route(x.cuda().bfloat16(), T, router.cuda(), k, True, cw, ids, wts)
    xb = x.bfloat16().float()
    for t in range(T):
        rid, rw = compute_routing(xb[t] @ router.t(), k)
        assert ids[t].tolist() == rid
        torch.testing.assert_close(wts[t].cpu(), rw, rtol=1e-4, atol=1e-5)
        dense = torch.zeros(E)
        dense[rid] = rw
        torch.testing.assert_close(cw[t].cpu(), dense, rtol=1e-4, atol=1e-5)


@pytest.mark.gpu
@pytest.mark.parametrize("qt", [GGMLType.Q8_0, GGMLType.Q4_K])
def test_moe_engine_matches_oracle(qt):
    from air_rs.runtime.builder import build_runner
    from air_rs.runtime.engine import Engine, SamplingParams
    from test_engine_gpu import _check_near_argmax
    cfg = tiny_moe()
    recs = list(random_tensors(cfg, qt, seed=0, device="cpu"))
    oracle = OracleModel(cfg, {n: (r, q, s) for n, r, q, s in recs})
    runner = build_runner(cfg, iter(recs), device="cuda", max_batch=16, max_model_len=512, num_blocks=512)
    runner.gemv_max_b = 8                 # 3 rows: the GEMV path; 12 rows: the GEMM path
    eng = Engine(cfg, runner, max_batch=16)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, cfg.vocab_size, (int(n),), generator=g).tolist() for n in (20, 33, 9)]
    outs = eng.generate_ids(prompts, SamplingParams(max_tokens=12, temperature=0.0, ignore_eos=True))
    for p, o in zip(prompts, outs):
        assert len(o) == 12
        _check_near_argmax(oracle, [cfg.bos_token_id] + p, o)
    # batched (GEMM path, 12 rows > 8)
    prompts = [torch.randint(0, cfg.vocab_size, (int(n),), generator=g).tolist() for n in range(5, 17)]
    outs = eng.generate_ids(prompts, SamplingParams(max_tokens=6, temperature=0.0, ignore_eos=True))
    _check_near_argmax(oracle, [cfg.bos_token_id] + prompts[0], outs[0])
    runner.check_errors()


@pytest.mark.gpu
def test_moe_select_gather_scatter_kernels():
    from air_rs import ops
    ext = ops.require_ext()
    g = torch.Generator().manual_seed(1)
    T, E, H = 300, 8, 256
    cw = torch.zeros(T, E)
    for t in range(T):
        e = torch.randperm(E, generator=g)[:2]
        cw[t, e] = torch.rand(2, generator=g) + 0.1
    cw = cw.cuda()
    idx = torch.zeros(T, dtype=torch.int32, device="cuda")
    wts = torch.zeros(T, device="cuda")
    cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
    ext.moe_select(cw, 3, T, idx, wts, cnt)
    want = torch.nonzero(cw[:, 3].cpu() > 0).flatten()
    n = int(cnt.item())
    assert n == want.numel() and idx[:n].cpu().tolist() == want.tolist()
    torch.testing.assert_close(wts[:n].cpu(), cw[want, 3].cpu())
    x = torch.randn(T, H, generator=g).cuda().bfloat16()
    xg = torch.zeros(T, H, device="cuda", dtype=torch.bfloat16)
    ext.moe_gather(x, idx, cnt, T, xg)
    assert torch.equal(xg[:n], x[want.cuda()])
    out = torch.zeros(T, H, device="cuda")
    y = torch.randn(T, H, generator=g).cuda()
    ext.moe_scatter(out, y, idx, wts, cnt, T)
    ref = torch.zeros(T, H)
    ref[want] = cw[want, 3].cpu()[:, None] * y[:n].cpu()
    torch.testing.assert_close(out.cpu(), ref)


@pytest.mark.gpu
def test_grouped_gemm_row_count_limits_work():
    from air_rs import ops
    from air_rs.ops import gemm
    from air_rs.gguf import quantize
    g = torch.Generator().manual_seed(2)
    N, K, T = 256, 512, 300
    w = ops.QWeight.from_raw(quantize(torch.randn(N, K, generator=g) * 0.05, GGMLType.Q4_K), GGMLType.Q4_K, N, K, "cuda")
    x = torch.randn(T, K, generator=g).cuda().bfloat16()
    full = torch.zeros(T, N, device="cuda")
    gemm.linear(x, w, full)
    part = torch.full((T, N), 7.0, device="cuda")
    gemm.linear(x, w, part, row_count=torch.tensor([40], dtype=torch.int32, device="cuda"))
    torch.testing.assert_close(part[:40], full[:40])
    assert torch.all(part[256:] == 7.0)     # token tiles (256 rows at T=300) past the count did nothing


@pytest.mark.gpu
@pytest.mark.parametrize("qt,E", [(GGMLType.Q4_K, 4), (GGMLType.Q8_0, 10)])
def test_grouped_expert_ffn_matches_per_expert_launches(monkeypatch, qt, E):
    """The grouped routed-expert path (grouped select / gather, one grouped GEMM per
    projection for up to 8 experts, grouped scatter) against one launch chain per expert."""
    from air_rs.models.config import tiny_moe
    from air_rs.parallel import moe
    from air_rs.runtime.builder import build_runner
    cfg = tiny_moe()
    cfg.n_experts = E
    recs = list(random_tensors(cfg, qt, seed=4, device="cpu"))
    rn = build_runner(cfg, iter(recs), device="cuda", max_batch=16, max_model_len=256, num_blocks=64)
    lw = rn.w.layers[0]
    assert moe._grouped_ok(rn, lw)
    g = torch.Generator().manual_seed(E)
    T = 37
    xn = (torch.randn(T, cfg.hidden_dim, generator=g)).to("cuda", torch.bfloat16)
    x0 = torch.randn(T, cfg.hidden_dim, generator=g).cuda()
    outs = {}
    for grouped in ("1", "0"):
        monkeypatch.setenv("AIR_MOE_GROUPED", grouped)
        x = x0.clone()
        moe.moe_ffn_prefill(rn, lw, T, x, xn)
        torch.cuda.synchronize()
        outs[grouped] = x
    rn.check_errors()
    torch.testing.assert_close(outs["1"], outs["0"], rtol=1e-4, atol=1e-4)
    assert not torch.equal(outs["1"], x0)
