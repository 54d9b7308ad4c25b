"""Architecture variants (reference src/model.rs:326-416, :623-660, src/model_variant.rs:140-189):
Qwen2 q/k/v biases, Gemma RMSNorm (weight + 1) + GeGLU + attention logit soft-capping, Falcon LayerNorm with biases + dense
GELU MLP, Phi-3 fused attn_qkv / [gate; up] tensors.

CPU: the reference-numerics oracle against a plain fp32 PyTorch forward written out here
from the definitions (dequantised weights), and GGUF round trips that recover the layout.
GPU (marked): the sm_100a engine against the oracle, decode GEMV path and batched GEMM path."""
import math

import pytest
import torch
import torch.nn.functional as F

from air_rs.gguf import GGMLType
from air_rs.gguf.quants import dequantize
from air_rs.models.config import FfnType, ModelConfig, NormType, tiny_variant
from air_rs.models.random_init import random_tensors, write_random_gguf
from air_rs.models.reference import OracleModel

ARCHS = ["qwen2", "gemma", "falcon", "phi3"]


def _deq(recs, name):
    raw, qt, shape = recs[name]
    return dequantize(raw.reshape(-1, raw.shape[-1]) if raw.dim() > 1 else raw.reshape(1, -1), qt).reshape(shape).float()


def _plain_forward(cfg: ModelConfig, recs: dict, ids: list[int]) -> torch.Tensor:
    """Logits of the last position, fp32 throughout, straight from the definitions."""
    H, nh, nkv, hd, Fd = cfg.hidden_dim, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.intermediate_dim
    w = lambda n: _deq(recs, n)
    has = lambda n: n in recs

    def norm(x, p):
        wt = w(p + ".weight")
        b = w(p + ".bias") if has(p + ".bias") else 0.0
        if cfg.norm_type == NormType.LAYER:
            return F.layer_norm(x, (H,), eps=cfg.rms_norm_eps) * wt + b
        if cfg.norm_type == NormType.GEMMA_RMS:
            wt = wt + 1.0
        return x * torch.rsqrt((x * x).mean(-1, keepdim=True) + cfg.rms_norm_eps) * wt + b

    def gelu(x):
        return F.gelu(x, approximate="tanh")

    S = len(ids)
    x = w("token_embd.weight")[torch.tensor(ids)]
    inv = 1.0 / cfg.rope_theta ** (torch.arange(0, hd, 2).float() / hd)
    ang = torch.arange(S).float()[:, None] * inv[None]
    cos, sin = torch.cos(ang)[:, None], torch.sin(ang)[:, None]

    def rope(t):
        a, b = t[..., : hd // 2], t[..., hd // 2:]
        return torch.cat([a * cos - b * sin, a * sin + b * cos], -1)

    for i in range(cfg.n_layers):
        p = f"blk.{i}."
        h = norm(x, p + "attn_norm")
        if has(p + "attn_qkv.weight"):
            wq, wk, wv = w(p + "attn_qkv.weight").split([nh * hd, nkv * hd, nkv * hd])
        else:
            wq, wk, wv = w(p + "attn_q.weight"), w(p + "attn_k.weight"), w(p + "attn_v.weight")
        q, k, v = h @ wq.t(), h @ wk.t(), h @ wv.t()
        if has(p + "attn_q.bias"):
            q, k, v = q + w(p + "attn_q.bias"), k + w(p + "attn_k.bias"), v + w(p + "attn_v.bias")
        q, k, v = rope(q.view(S, nh, hd)), rope(k.view(S, nkv, hd)), v.view(S, nkv, hd)
        rep = nh // nkv
        k, v = k.repeat_interleave(rep, 1), v.repeat_interleave(rep, 1)
        sc = (q.transpose(0, 1) @ k.transpose(0, 1).transpose(-1, -2)) / math.sqrt(hd)   # [h, S, S]
        if cfg.attn_softcap > 0:
            sc = cfg.attn_softcap * torch.tanh(sc / cfg.attn_softcap)
        sc = sc.masked_fill(torch.triu(torch.ones(S, S, dtype=torch.bool), 1)[None], float("-inf"))
        a = (torch.softmax(sc, -1) @ v.transpose(0, 1)).transpose(0, 1).reshape(S, nh * hd)
        x = x + a @ w(p + "attn_output.weight").t()
        h = norm(x, p + "ffn_norm")
        if cfg.ffn_type == FfnType.DENSE:
            m = gelu(h @ w(p + "ffn_up.weight").t())
        else:
            if has(p + "ffn_gate.weight"):
                g, u = h @ w(p + "ffn_gate.weight").t(), h @ w(p + "ffn_up.weight").t()
            else:
                g, u = (h @ w(p + "ffn_up.weight").t()).split([Fd, Fd], -1)
            m = (gelu(g) if cfg.ffn_type == FfnType.GEGLU else F.silu(g)) * u
        x = x + m @ w(p + "ffn_down.weight").t()
    x = norm(x, "output_norm")
    return x[-1] @ w("output.weight").t()


@pytest.mark.parametrize("arch", ARCHS)
def test_oracle_matches_plain_forward(arch):
    cfg = tiny_variant(arch)
    recs = {n: (r, q, s) for n, r, q, s in random_tensors(cfg, GGMLType.Q8_0, seed=1, device="cpu")}
    ids = torch.randint(3, cfg.vocab_size, (12,), generator=torch.Generator().manual_seed(2)).tolist()
    ref = _plain_forward(cfg, recs, ids)
    got = OracleModel(cfg, recs).forward(ids, 0)
    # the oracle quantises activations (Q8_0) and keeps an F16 residual stream
    cos = F.cosine_similarity(got, ref, dim=0)
    assert cos > 0.999, float(cos)
    assert float((got - ref).abs().max()) < 0.05 * float(ref.max() - ref.min())


@pytest.mark.parametrize("arch", ARCHS)
def test_variant_gguf_roundtrip_layout(tmp_path, arch):
    from air_rs.gguf import read_gguf
    cfg = tiny_variant(arch)
    path = write_random_gguf(str(tmp_path / f"{arch}.gguf"), cfg, GGMLType.Q8_0, seed=0)
    g = read_gguf(path)
    back = ModelConfig.from_gguf_metadata(g.metadata).detect_layout(g.tensors)
    for f in ("qkv_bias", "norm_bias", "fused_qkv", "fused_gate_up", "norm_type", "ffn_type", "attn_softcap"):
        assert getattr(back, f) == getattr(cfg, f), f
    o1 = OracleModel.from_gguf(g).forward([5, 6, 7], 0)
    recs = {n: (r, q, s) for n, r, q, s in random_tensors(cfg, GGMLType.Q8_0, seed=0, device="cpu")}
    torch.testing.assert_close(o1, OracleModel(cfg, recs).forward([5, 6, 7], 0))
    g.close()


@pytest.mark.gpu
@pytest.mark.parametrize("arch", ARCHS)
@pytest.mark.parametrize("qt", [GGMLType.Q4_K, GGMLType.Q8_0])
def test_engine_variant_matches_oracle(arch, qt):
    from air_rs.models.reference import apply_repetition_penalty
    from air_rs.runtime.builder import build_runner
    from air_rs.runtime.engine import Engine, SamplingParams
    cfg = tiny_variant(arch)
    recs = list(random_tensors(cfg, qt, seed=0, device="cpu"))
    oracle = OracleModel(cfg, {n: (r, q, s) for n, r, q, s in recs})
    runner = build_runner(cfg, iter(recs), device="cuda", max_batch=16, max_model_len=256, num_blocks=256)
    eng = Engine(cfg, runner, max_batch=16)
    g = torch.Generator().manual_seed(3)
    # one prompt alone (decode GEMV path), then 12 together (batched GEMM path)
    for n in (1, 12):
        prompts = [torch.randint(3, cfg.vocab_size, (int(l),), generator=g).tolist()
                   for l in torch.randint(5, 40, (n,), generator=g)]
        outs = eng.generate_ids(prompts, SamplingParams(max_tokens=8, temperature=0.0, ignore_eos=True))
        runner.check_errors()
        for p, toks in list(zip(prompts, outs))[:3]:
            oracle.reset()
            seq = [cfg.bos_token_id] + p
            logits = oracle.forward(seq, 0)
            for t in toks:
                lg = apply_repetition_penalty(logits, seq, 1.1)
                assert float(lg.max() - lg[t]) <= 0.15 * float(lg.max() - lg.min()), (arch, n, t)
                seq.append(t)
                logits = oracle.forward([t], len(seq) - 1)
