"""FP8 (E4M3) paged KV pool: the row format on the host, sizing and configuration (CPU), and
the writer / attention kernels and the engine on it (GPU, against fp32 references)."""
import pytest
import torch

from air_rs.config import EngineConfig
from air_rs.kv.fp8 import dequantize_rows, quantize_rows, row_bytes
from air_rs.kv.prefix_store import PrefixKvStore
from air_rs.models.config import tiny_llama
from air_rs.runtime.builder import kv_bytes_per_block, kv_row_bytes


def test_row_format_round_trip():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(4, 3, 128, generator=g) * torch.tensor([0.01, 1.0, 300.0]).view(1, 3, 1)
    q = quantize_rows(x)
    assert q.dtype == torch.uint8 and q.shape == (4, 3, row_bytes(128)) and row_bytes(128) % 16 == 0
    assert torch.all(q[..., 132:] == 0)                  # padding
    s = q[..., 128:132].contiguous().view(torch.float32).squeeze(-1)
    torch.testing.assert_close(s, x.abs().amax(-1) / 448.0)
    y = dequantize_rows(q)
    # E4M3 has 3 mantissa bits: relative error <= 2^-4 of each value (plus underflow near 0)
    err = (y - x).abs()
    assert torch.all(err <= x.abs() * 2 ** -4 + s.unsqueeze(-1) * 2 ** -9 + 1e-12)
    # the largest element of each row is exact (code 448)
    i = x.abs().argmax(-1, keepdim=True)
    torch.testing.assert_close(y.gather(-1, i), x.gather(-1, i), rtol=1e-6, atol=0)


def test_zero_row_and_sizes():
    z = dequantize_rows(quantize_rows(torch.zeros(2, 64)))
    assert torch.all(z == 0)
    cfg = tiny_llama()
    assert kv_row_bytes(128, "fp8") == 144 and kv_row_bytes(128) == 256
    bf, f8 = kv_bytes_per_block(cfg, 16), kv_bytes_per_block(cfg, 16, kv_dtype="fp8")
    assert f8 * cfg.head_dim * 2 == bf * (cfg.head_dim + 16)
    with pytest.raises(ValueError):
        kv_row_bytes(128, "int4")


def test_engine_config_kv_dtype():
    assert EngineConfig.from_env({"AIR_KV_DTYPE": "fp8"}, preset="tiny").kv_dtype == "fp8"
    with pytest.raises(ValueError):
        EngineConfig.from_env({"AIR_KV_DTYPE": "fp4"}, preset="tiny")


def test_prefix_store_keeps_fp8_rows_raw():
    kv = quantize_rows(torch.randn(2, 6, 2, 2, 4, 64))      # [L, blocks, 2, nkv, bs, 80]
    st = PrefixKvStore()
    st.store("m", kv, [3, 1], list(range(7)))
    with pytest.raises(ValueError):
        st.store("m", kv, [3, 1], list(range(7)), scheme="q8")
    from air_rs.kv.prefix_store import _decode
    got = _decode(st._e["m"])
    assert got.dtype == torch.uint8 and torch.equal(got, kv[:, [3, 1]])


# ------------------------------------------------------------------------------- GPU
def _paged_fp8(lens, nkv, d, bs, seed=0):
    from tests.test_kernels_gpu import _paged_setup
    kv, bt, _ = _paged_setup(lens, nkv, d, bs, seed)
    kv8 = quantize_rows(kv.float() * 3.0)
    deq = dequantize_rows(kv8)
    dense = []
    for i, l in enumerate(lens):
        ids = [int(b) for b in bt[i] if b >= 0]
        k = torch.cat([deq[b, 0].permute(1, 0, 2) for b in ids], 0)[:l]
        v = torch.cat([deq[b, 1].permute(1, 0, 2) for b in ids], 0)[:l]
        dense.append((k, v))
    return kv8, bt, dense


@pytest.mark.gpu
@pytest.mark.parametrize("d,G", [(128, 1), (128, 4), (128, 8), (64, 4)])
@pytest.mark.parametrize("splits", [1, 5])
def test_fp8_decode_attention(d, G, splits):
    """Decode rows on an fp8 pool (tensor-core kernel for head_dim 128, SIMT kernel for 64)
    against fp32 attention over the dequantised rows."""
    from air_rs import ops
    from air_rs.models.reference import attention_reference
    nkv, bs = 2, 16
    nh = nkv * G
    lens = [1, 40, 333, 900]
    kv8, bt, dense = _paged_fp8(lens, nkv, d, bs, seed=2)
    R = len(lens)
    q = torch.randn(R, nh, d, generator=torch.Generator().manual_seed(9))
    out = torch.zeros(R, nh, d, device="cuda")
    part_o = torch.zeros(R * nh * splits * d, device="cuda")
    part_ml = torch.zeros(R * nh * splits * 2, device="cuda")
    ops.paged_attention(q.cuda(), kv8.cuda(), bt.cuda(), torch.tensor(lens, dtype=torch.int32, device="cuda"),
                        out, n_rows=R, n_heads=nh, n_kv=nkv, head_dim=d, block_size=bs, n_splits=splits,
                        split_tokens=0, part_o=part_o, part_ml=part_ml)
    for i in range(R):
        ref = attention_reference(q[i:i + 1], dense[i][0], dense[i][1], causal=False)[0]
        torch.testing.assert_close(out[i].cpu(), ref, rtol=1e-2, atol=1e-2)


@pytest.mark.gpu
@pytest.mark.parametrize("G", [1, 4, 8])
def test_fp8_prefill_attention(G):
    """Query-tiled prefill kernel on an fp8 pool (rows of three sequences, causal)."""
    from air_rs import ops
    from air_rs.models.reference import attention_reference
    nkv, d, bs = 2, 128, 16
    nh = nkv * G
    lens, qlen = [75, 130, 33], [40, 130, 21]
    kv8, bt, dense = _paged_fp8(lens, nkv, d, bs, seed=4)
    rows_seq, ctx = [], []
    for s_, (L, n) in enumerate(zip(lens, qlen)):
        rows_seq += [s_] * n
        ctx += list(range(L - n + 1, L + 1))
    T = len(rows_seq)
    q = torch.randn(T, nh, d, generator=torch.Generator().manual_seed(3))
    out = torch.zeros(T, nh, d, device="cuda")
    ops.paged_attention(q.cuda(), kv8.cuda(), bt.cuda(), torch.tensor(ctx, dtype=torch.int32, device="cuda"),
                        out, n_rows=T, n_heads=nh, n_kv=nkv, head_dim=d, block_size=bs,
                        row_seq=torch.tensor(rows_seq, dtype=torch.int32, device="cuda"))
    torch.cuda.synchronize()
    r = 0
    for s_, (L, n) in enumerate(zip(lens, qlen)):
        k, v = dense[s_]
        ref = attention_reference(q[r:r + n], k, v, causal=True)
        torch.testing.assert_close(out[r:r + n].cpu(), ref, rtol=1e-2, atol=1e-2)
        r += n


@pytest.mark.gpu
@pytest.mark.parametrize("d", [64, 128])
def test_fp8_rope_kv_writer(d):
    """rope_kv into an fp8 pool: Q rows as in the bf16 path, K/V rows equal to the host
    quantisation of the fp32 RoPE'd values (scale to rounding, codes within one step)."""
    from air_rs import ops
    from tests.test_kernels_gpu import _rope_ref
    T, nh, nkv, bs = 5, 4, 2, 16
    g = torch.Generator().manual_seed(1)
    qkv = torch.randn(T, (nh + 2 * nkv) * d, generator=g) * 4
    pos = torch.tensor([0, 3, 17, 64, 200], dtype=torch.int32)
    slots = torch.tensor([0, 17, 33, 2, -1], dtype=torch.int64)
    cs = ops.rope_table(256, d, 10000.0, "cuda")
    kv = torch.zeros(4, 2, nkv, bs, d + 16, dtype=torch.uint8, device="cuda")
    q = torch.zeros(T, nh, d, device="cuda")
    ops.rope_kv(qkv.cuda(), T, cs, pos.cuda(), slots.cuda(), kv, q, n_heads=nh, n_kv=nkv, head_dim=d,
                block_size=bs)
    torch.cuda.synchronize()
    qr = _rope_ref(qkv[:, :nh * d].reshape(T, nh, d), pos, 10000.0, d)
    kr = _rope_ref(qkv[:, nh * d:(nh + nkv) * d].reshape(T, nkv, d), pos, 10000.0, d)
    vr = qkv[:, (nh + nkv) * d:].reshape(T, nkv, d)
    torch.testing.assert_close(q.cpu(), qr, rtol=1e-4, atol=1e-4)
    kvc = kv.cpu()
    for t in range(T):
        if slots[t] < 0:
            continue
        blk, off = int(slots[t]) // bs, int(slots[t]) % bs
        for which, ref in ((0, kr[t]), (1, vr[t])):
            row = kvc[blk, which, :, off]                      # [nkv, d + 16]
            want = quantize_rows(ref)
            torch.testing.assert_close(row[:, d:d + 4].contiguous().view(torch.float32),
                                       want[:, d:d + 4].contiguous().view(torch.float32), rtol=1e-4, atol=0)
            torch.testing.assert_close(dequantize_rows(row), ref, rtol=7e-2, atol=ref.abs().max().item() / 448)


@pytest.mark.gpu
def test_engine_fp8_kv_matches_oracle():
    """Greedy decode on an fp8 KV pool (GEMV decode path and tensor-core GEMM prefill) stays
    at the oracle's argmax under teacher forcing, like the bf16 pool."""
    from air_rs.gguf import GGMLType
    from air_rs.models.random_init import random_tensors
    from air_rs.models.reference import OracleModel
    from air_rs.runtime.builder import build_runner
    from air_rs.runtime.engine import Engine, SamplingParams
    from tests.test_engine_gpu import _check_near_argmax
    cfg = tiny_llama()
    recs = list(random_tensors(cfg, GGMLType.Q8_0, seed=0, device="cpu"))
    oracle = OracleModel(cfg, {n: (r, q, s) for n, r, q, s in recs})
    runner = build_runner(cfg, iter(recs), device="cuda", max_batch=16, max_model_len=512, num_blocks=256,
                          kv_dtype="fp8")
    assert runner.kv.dtype == torch.uint8 and runner.kv.shape[-1] == cfg.head_dim + 16
    runner.gemv_max_b = 8                 # decode through the GEMV -> rope_kv path
    eng = Engine(cfg, runner, max_batch=16)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (32, 50, 7)]
    outs = eng.generate_ids(prompts, SamplingParams(max_tokens=16, temperature=0.0, ignore_eos=True))
    for p, o in zip(prompts, outs):
        assert len(o) == 16
        _check_near_argmax(oracle, [cfg.bos_token_id] + p, o, tol=0.2)
    runner.gemv_max_b = 1                 # and through the tensor-core GEMM step
    runner.graphs.clear()
    outs = eng.generate_ids(prompts, SamplingParams(max_tokens=16, temperature=0.0, ignore_eos=True))
    for p, o in zip(prompts, outs):
        _check_near_argmax(oracle, [cfg.bos_token_id] + p, o, tol=0.2)
    runner.check_errors()
