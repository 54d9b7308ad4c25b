"""Numerics of the sm_100a kernels against plain PyTorch fp32 references."""
import math

import pytest
import torch

from air_rs import ops
from air_rs.gguf import GGMLType, quantize, dequantize
from air_rs.models.reference import attention_reference

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _qw(N, K, qt, seed=0):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(N, K, generator=g) * 0.02
    raw = quantize(w, qt)
    wd = dequantize(raw, qt).reshape(N, K)
    return ops.QWeight.from_raw(raw, qt, N, K, DEV), wd


def _act(B, K, seed=1):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(B, K, generator=g)


def _quant_act_ref(x):
    xb = x.reshape(x.shape[0], -1, 32)
    d = xb.abs().amax(-1, keepdim=True) / 127.0
    q = torch.where(d > 0, torch.round(xb / d), torch.zeros_like(xb)).clamp(-127, 127)
    return (q * d).reshape(x.shape)


@pytest.mark.parametrize("qt", [GGMLType.Q4_K, GGMLType.Q8_0, GGMLType.F16])
@pytest.mark.parametrize("B", [1, 3, 8])
def test_gemv_store(qt, B):
    N, K = 384, 1024
    w, wd = _qw(N, K, qt)
    x = _act(B, K)
    xg = x.to(DEV)
    xq = torch.empty(B, K, dtype=torch.int8, device=DEV)
    xds = torch.empty(B, K // 32, 2, dtype=torch.float32, device=DEV)
    ops.rmsnorm_quant(xg, None, 0.0, xq, xds)
    out = torch.zeros(B, N, device=DEV)
    ops.gemv(w, xq, xds, B, ops.EPI_STORE, out_f32=out)
    ref = _quant_act_ref(x) @ wd.t()
    if w.fmt == ops.FMT_BF16:
        ref = _quant_act_ref(x) @ wd.bfloat16().float().t()
    torch.testing.assert_close(out.cpu(), ref, rtol=2e-3, atol=2e-4)


@pytest.mark.parametrize("N,K", [(8192, 3072), (1280, 4096), (128, 256), (1000, 2048), (4096, 14336)])
@pytest.mark.parametrize("B", [1, 5])
def test_gemv_q4k_stream_k_shapes(N, K, B):
    """Persistent GEMV: CTA ranges that start and end inside tiles, tiles completed by one
    CTA, a single-unit grid, a partial last tile; the same launch twice (self-resetting
    tile counters)."""
    w, wd = _qw(N, K, GGMLType.Q4_K)
    x = _act(B, K)
    xq = torch.empty(B, K, dtype=torch.int8, device=DEV)
    xds = torch.empty(B, K // 32, 2, dtype=torch.float32, device=DEV)
    ops.rmsnorm_quant(x.to(DEV), None, 0.0, xq, xds)
    ref = _quant_act_ref(x) @ wd.t()
    for _ in range(2):
        out = torch.full((B, N), float("nan"), device=DEV)
        ops.gemv(w, xq, xds, B, ops.EPI_STORE, out_f32=out)
        torch.testing.assert_close(out.cpu(), ref, rtol=2e-3, atol=float(ref.abs().max()) * 2e-4)


def test_rmsnorm_quant_matches():
    B, K = 4, 4096
    x = _act(B, K) * 3
    w = torch.rand(K) + 0.5
    xq = torch.empty(B, K, dtype=torch.int8, device=DEV)
    xds = torch.empty(B, K // 32, 2, dtype=torch.float32, device=DEV)
    y = torch.empty(B, K, dtype=torch.bfloat16, device=DEV)
    ops.rmsnorm_quant(x.to(DEV), w.to(DEV), 1e-5, xq, xds, y_bf16=y)
    ref = x / torch.sqrt((x * x).mean(-1, keepdim=True) + 1e-5) * w
    torch.testing.assert_close(y.float().cpu(), ref, rtol=1e-2, atol=1e-2)
    deq = (xq.float() .reshape(B, -1, 32) * xds[..., 0:1]).reshape(B, K).cpu()
    torch.testing.assert_close(deq, ref, rtol=0, atol=float(ref.abs().max()) / 120)
    s = xq.float().reshape(B, -1, 32).sum(-1) * xds[..., 0]
    torch.testing.assert_close(xds[..., 1], s)


@pytest.mark.parametrize("B,K", [(5, 4096), (37, 4096), (20, 2560), (16, 8192)])
@pytest.mark.parametrize("mode", ["rms", "layer_bias", "bf16_in", "no_w"])
def test_rmsnorm_quant_row_and_slice_kernels(B, K, mode):
    """Both launch shapes (B < 16: row slices over several CTAs; B >= 16: one CTA per row held
    in registers) against fp32 RMSNorm / LayerNorm (+ weight offset, bias) and the Q8A rule."""
    g = torch.Generator().manual_seed(B + K)
    x = torch.randn(B, K, generator=g) * 2 + (0.7 if mode == "layer_bias" else 0.0)
    w = torch.rand(K, generator=g) + 0.5
    bias = torch.randn(K, generator=g) * 0.1 if mode == "layer_bias" else None
    xq = torch.empty(B, K, dtype=torch.int8, device=DEV)
    xds = torch.empty(B, K // 32, 2, dtype=torch.float32, device=DEV)
    y = torch.empty(B, K, dtype=torch.bfloat16, device=DEV)
    kw = dict(y_bf16=y, bias=bias.to(DEV) if bias is not None else None, layer=mode == "layer_bias",
              w_offset=1.0 if mode == "rms" else 0.0)
    if mode == "bf16_in":
        x = x.bfloat16().float()
        ops.rmsnorm_quant(None, w.to(DEV), 1e-5, xq, xds, x_bf16=x.bfloat16().to(DEV), **kw)
    else:
        ops.rmsnorm_quant(x.to(DEV), None if mode == "no_w" else w.to(DEV), 1e-5, xq, xds, **kw)
    if mode == "no_w":
        ref = x
    elif mode == "layer_bias":
        c = x - x.mean(-1, keepdim=True)
        ref = c / torch.sqrt((c * c).mean(-1, keepdim=True) + 1e-5) * w + bias
    else:
        ref = x / torch.sqrt((x * x).mean(-1, keepdim=True) + 1e-5) * (w + kw["w_offset"])
    torch.testing.assert_close(y.float().cpu(), ref, rtol=1e-2, atol=1e-2)
    deq = (xq.float().reshape(B, -1, 32) * xds[..., 0:1]).reshape(B, K).cpu()
    torch.testing.assert_close(deq, _quant_act_ref(ref), rtol=0, atol=float(ref.abs().max()) / 120)
    s = xq.float().reshape(B, -1, 32).sum(-1) * xds[..., 0]
    torch.testing.assert_close(xds[..., 1], s)


def test_gemv_residual_and_swiglu():
    B, H, F = 2, 512, 768
    wg, wgd = _qw(F, H, GGMLType.Q4_K, 3)
    wu, wud = _qw(F, H, GGMLType.Q4_K, 4)
    x = _act(B, H)
    xq = torch.empty(B, H, dtype=torch.int8, device=DEV)
    xds = torch.empty(B, H // 32, 2, dtype=torch.float32, device=DEV)
    ops.rmsnorm_quant(x.to(DEV), None, 0, xq, xds)
    wgu = ops.QWeight.cat([wg, wu])
    h = torch.zeros(B, F, device=DEV)
    ops.gemv(wgu.rows(0, F), xq, xds, B, ops.EPI_SWIGLU, w2=wgu.rows(F, 2 * F), out_f32=h)
    xa = _quant_act_ref(x)
    g, u = xa @ wgd.t(), xa @ wud.t()
    torch.testing.assert_close(h.cpu(), g / (1 + torch.exp(-g)) * u, rtol=3e-3, atol=3e-5)
    wd, wdd = _qw(H, F, GGMLType.Q4_K, 5)
    hq = torch.empty(B, F, dtype=torch.int8, device=DEV)
    hds = torch.empty(B, F // 32, 2, dtype=torch.float32, device=DEV)
    ops.rmsnorm_quant(h, None, 0, hq, hds)
    resid = torch.ones(B, H, device=DEV)
    ops.gemv(wd, hq, hds, B, ops.EPI_RESIDUAL, resid=resid)
    ref = 1 + _quant_act_ref(h.cpu()) @ wdd.t()
    torch.testing.assert_close(resid.cpu(), ref, rtol=2e-3, atol=1e-5)


@pytest.mark.parametrize("B", [1, 3, 8])
def test_gemv_swiglu_quantised_epilogue_matches_separate_quant(B):
    """SwiGLU GEMV writing its product as Q8A (int8 + per-32 scales) equals the GEMV's fp32
    output quantised by rmsnorm_quant, element for element; padded rows N..q_k are zero."""
    H, F, Fp = 1024, 1200, 1216
    wg, _ = _qw(F, H, GGMLType.Q4_K, 6)
    wu, _ = _qw(F, H, GGMLType.Q4_K, 7)
    x = _act(B, H, seed=2)
    xq = torch.empty(B, H, dtype=torch.int8, device=DEV)
    xds = torch.empty(B, H // 32, 2, dtype=torch.float32, device=DEV)
    ops.rmsnorm_quant(x.to(DEV), None, 0, xq, xds)
    h = torch.zeros(B, Fp, device=DEV)
    ops.gemv(wg, xq, xds, B, ops.EPI_SWIGLU, w2=wu, out_f32=h, ld_out=Fp)
    rq = torch.empty(B, Fp, dtype=torch.int8, device=DEV)
    rds = torch.empty(B, Fp // 32, 2, dtype=torch.float32, device=DEV)
    ops.rmsnorm_quant(h, None, 0, rq, rds)
    hq = torch.full((B, Fp), 99, dtype=torch.int8, device=DEV)
    hds = torch.full((B, Fp // 32, 2), float("nan"), device=DEV)
    ops.gemv(wg, xq, xds, B, ops.EPI_SWIGLU, w2=wu, ld_out=Fp, out_q=hq, out_ds=hds)
    assert torch.equal(hq.cpu(), rq.cpu())
    torch.testing.assert_close(hds.cpu(), rds.cpu(), rtol=0, atol=0)
    assert (hq[:, F:] == 0).all()


def _rope_ref(x, pos, theta, d):
    inv = 1.0 / torch.pow(torch.tensor(theta), torch.arange(0, d, 2, dtype=torch.float32) / d)
    ang = pos[:, None].float() * inv[None]
    c, s = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]
    h = d // 2
    return torch.cat([x[..., :h] * c - x[..., h:] * s, x[..., :h] * s + x[..., h:] * c], -1)


def test_gemv_qkv_rope_kv_write():
    B, H, nh, nkv, d, bs = 3, 512, 4, 2, 128, 16
    N = (nh + 2 * nkv) * d
    w, wd = _qw(N, H, GGMLType.Q4_K, 7)
    x = _act(B, H)
    xq = torch.empty(B, H, dtype=torch.int8, device=DEV)
    xds = torch.empty(B, H // 32, 2, dtype=torch.float32, device=DEV)
    ops.rmsnorm_quant(x.to(DEV), None, 0, xq, xds)
    kv = torch.zeros(8, 2, nkv, bs, d, dtype=torch.bfloat16, device=DEV)
    pos = torch.tensor([0, 17, 100], dtype=torch.int32)
    slots = torch.tensor([5, 3 * bs + 1, 7 * bs + 4], dtype=torch.int64)
    cs = ops.rope_table(256, d, 10000.0, DEV)
    q = torch.zeros(B, nh, d, device=DEV)
    ops.gemv(w, xq, xds, B, ops.EPI_QKV_ROPE, rope_cs=cs, positions=pos.to(DEV), slots=slots.to(DEV),
             kv=kv, q_out=q, n_heads=nh, n_kv=nkv, head_dim=d, block_size=bs)
    y = _quant_act_ref(x) @ wd.t()
    qr = _rope_ref(y[:, :nh * d].reshape(B, nh, d), pos, 10000.0, d)
    kr = _rope_ref(y[:, nh * d:(nh + nkv) * d].reshape(B, nkv, d), pos, 10000.0, d)
    vr = y[:, (nh + nkv) * d:].reshape(B, nkv, d)
    torch.testing.assert_close(q.cpu(), qr, rtol=3e-3, atol=1e-4)
    kvc = kv.float().cpu()
    for b in range(B):
        blk, off = int(slots[b]) // bs, int(slots[b]) % bs
        torch.testing.assert_close(kvc[blk, 0, :, off], kr[b], rtol=1e-2, atol=1e-3)
        torch.testing.assert_close(kvc[blk, 1, :, off], vr[b], rtol=1e-2, atol=1e-3)


def _paged_setup(lens, nkv, d, bs, seed=0):
    g = torch.Generator().manual_seed(seed)
    nblocks = sum((l + bs - 1) // bs for l in lens) + 4
    kv = torch.randn(nblocks, 2, nkv, bs, d, generator=g).bfloat16()
    perm = torch.randperm(nblocks, generator=g).tolist()
    maxb = max((l + bs - 1) // bs for l in lens)
    bt = torch.full((len(lens), maxb), -1, dtype=torch.int32)
    dense = []
    p = 0
    for i, l in enumerate(lens):
        nb = (l + bs - 1) // bs
        ids = perm[p:p + nb]
        p += nb
        bt[i, :nb] = torch.tensor(ids, dtype=torch.int32)
        k = torch.cat([kv[b, 0].permute(1, 0, 2) for b in ids], 0)[:l]  # [l, nkv, d]
        v = torch.cat([kv[b, 1].permute(1, 0, 2) for b in ids], 0)[:l]
        dense.append((k.float(), v.float()))
    return kv, bt, dense


@pytest.mark.parametrize("splits", [1, 4, 13])
@pytest.mark.parametrize("G", [1, 4, 8])
@pytest.mark.parametrize("cap", [0.0, 3.0])
def test_paged_decode_attention(splits, G, cap):
    nkv, d, bs = 2, 128, 16
    nh = nkv * G
    lens = [1, 37, 300, 1000]
    kv, bt, dense = _paged_setup(lens, nkv, d, bs)
    R = len(lens)
    q = torch.randn(R, nh, d, generator=torch.Generator().manual_seed(5))
    out = torch.zeros(R, nh, d, device=DEV)
    part_o = torch.zeros(R * nh * splits * d, device=DEV)
    part_ml = torch.zeros(R * nh * splits * 2, device=DEV)
    ops.paged_attention(q.to(DEV), kv.to(DEV), bt.to(DEV), torch.tensor(lens, dtype=torch.int32, device=DEV),
                        out, n_rows=R, n_heads=nh, n_kv=nkv, head_dim=d, block_size=bs,
                        n_splits=splits, split_tokens=0, part_o=part_o, part_ml=part_ml, softcap=cap)
    for i, l in enumerate(lens):
        ref = attention_reference(q[i:i + 1], dense[i][0], dense[i][1], causal=False, softcap=cap)[0]
        # tensor-core path: Q and P enter the MMA as bf16
        torch.testing.assert_close(out[i].cpu(), ref, rtol=1e-2, atol=8e-3)


def test_paged_prefill_causal_and_tree():
    nkv, G, d, bs = 2, 4, 64, 16
    nh = nkv * G
    L = 70
    kv, bt, dense = _paged_setup([L], nkv, d, bs, seed=3)
    T = 20  # last T tokens are queries at positions L-T .. L-1
    q = torch.randn(T, nh, d)
    ctx = torch.arange(L - T + 1, L + 1, dtype=torch.int32)
    out = torch.zeros(T, nh, d, device=DEV)
    ops.paged_attention(q.to(DEV), kv.to(DEV), bt.to(DEV), ctx.to(DEV), out, n_rows=T, n_heads=nh,
                        n_kv=nkv, head_dim=d, block_size=bs,
                        row_seq=torch.zeros(T, dtype=torch.int32, device=DEV))
    ref = attention_reference(q, dense[0][0], dense[0][1], causal=True)
    torch.testing.assert_close(out.cpu(), ref, rtol=2e-3, atol=2e-3)
    # tree: queries are the last T tokens; each sees the prefix plus its ancestors
    base = L - T
    parents = [-1] + [max(-1, (i - 1) // 2) for i in range(1, T)]
    masks, dense_mask = [], torch.zeros(T, L, dtype=torch.bool)
    for i in range(T):
        m, j = 0, i
        while j >= 0:
            m |= 1 << j
            j = parents[j]
        masks.append(m)
        dense_mask[i, :base] = True
        for j in range(T):
            if (m >> j) & 1:
                dense_mask[i, base + j] = True
    tm = torch.tensor([m if m < 2**63 else m - 2**64 for m in masks], dtype=torch.int64)
    out2 = torch.zeros_like(out)
    ops.paged_attention(q.to(DEV), kv.to(DEV), bt.to(DEV), torch.full((T,), L, dtype=torch.int32, device=DEV),
                        out2, n_rows=T, n_heads=nh, n_kv=nkv, head_dim=d, block_size=bs,
                        row_seq=torch.zeros(T, dtype=torch.int32, device=DEV),
                        tree_base=torch.full((T,), base, dtype=torch.int32, device=DEV),
                        tree_mask=tm.to(DEV))
    ref2 = attention_reference(q, dense[0][0], dense[0][1], causal=False, mask=dense_mask)
    torch.testing.assert_close(out2.cpu(), ref2, rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("G", [1, 2, 4, 8])
@pytest.mark.parametrize("window,cap", [(0, 0.0), (50, 0.0), (0, 3.0)])
def test_query_tiled_prefill_attention(G, window, cap):
    """The query-tiled prefill kernel (16 rows per CTA, shared K/V tiles) against dense fp32
    attention: three sequences whose chunks straddle 16-row tiles (mixed-sequence tiles),
    chunked prefill (queries start mid-sequence), GQA groups 1-8, sliding window."""
    nkv, d, bs = 2, 128, 16
    nh = nkv * G
    lens = [75, 130, 33]          # total keys per sequence
    qlen = [40, 130, 21]          # the last qlen tokens of each are this step's queries
    kv, bt, dense = _paged_setup(lens, nkv, d, bs, seed=7)
    rows_seq, ctx = [], []
    for s_, (L, n) in enumerate(zip(lens, qlen)):
        rows_seq += [s_] * n
        ctx += list(range(L - n + 1, L + 1))
    T = len(rows_seq)
    q = torch.randn(T, nh, d, generator=torch.Generator().manual_seed(11))
    out = torch.zeros(T, nh, d, device=DEV)
    ops.paged_attention(q.to(DEV), kv.to(DEV), bt.to(DEV), torch.tensor(ctx, dtype=torch.int32, device=DEV), out,
                        n_rows=T, n_heads=nh, n_kv=nkv, head_dim=d, block_size=bs,
                        row_seq=torch.tensor(rows_seq, dtype=torch.int32, device=DEV), window=window,
                        softcap=cap)
    torch.cuda.synchronize()
    r = 0
    for s_, (L, n) in enumerate(zip(lens, qlen)):
        k, v = dense[s_]
        mask = torch.zeros(n, L, dtype=torch.bool)
        for i in range(n):
            c = L - n + 1 + i
            lo = max(0, c - window) if window else 0
            mask[i, lo:c] = True
        ref = attention_reference(q[r:r + n], k, v, causal=False, mask=mask, softcap=cap)
        torch.testing.assert_close(out[r:r + n].cpu(), ref, rtol=1e-2, atol=8e-3)
        r += n


def test_sampler_greedy_penalty_and_topk():
    B, V = 3, 50000
    g = torch.Generator().manual_seed(0)
    logits = torch.randn(B, V, generator=g)
    counts = torch.zeros(4, V, dtype=torch.uint8)
    top = logits.argmax(-1)
    counts[1, top[1]] = 3  # penalise row 1's argmax
    toks = torch.zeros(B, dtype=torch.int32, device=DEV)
    ops.sample(logits.to(DEV), toks, counts=counts.to(DEV),
               count_row=torch.tensor([0, 1, 2], dtype=torch.int32, device=DEV),
               temperature=torch.zeros(B, device=DEV), penalty=torch.full((B,), 1.1, device=DEV))
    ref = logits.clone()
    v = ref[1, top[1]]
    ref[1, top[1]] = v / 1.1 ** 3 if v > 0 else v * 1.1 ** 3
    assert toks.cpu().tolist() == ref.argmax(-1).tolist()
    # top-k = 1 with temperature behaves like greedy
    ops.sample(logits.to(DEV), toks, temperature=torch.ones(B, device=DEV),
               top_k=torch.ones(B, dtype=torch.int32, device=DEV), top_p=torch.ones(B, device=DEV))
    assert toks.cpu().tolist() == logits.argmax(-1).tolist()
    # distribution check on a tiny vocab: sampled frequencies follow softmax within top-k
    V2, N = 8, 4000
    lg = torch.tensor([[2.0, 1.0, 0.5, 0.0, -1.0, -2.0, -3.0, -4.0]] * N)
    t2 = torch.zeros(N, dtype=torch.int32, device=DEV)
    ops.sample(lg.to(DEV), t2, temperature=torch.ones(N, device=DEV),
               top_k=torch.full((N,), 3, dtype=torch.int32, device=DEV), top_p=torch.ones(N, device=DEV),
               seed=123, step=torch.zeros(1, dtype=torch.int64, device=DEV))
    freq = torch.bincount(t2.cpu().long(), minlength=V2).float() / N
    p = torch.softmax(lg[0, :3], 0)
    assert freq[3:].sum() == 0
    torch.testing.assert_close(freq[:3], p, atol=0.04, rtol=0)


def test_embed_and_dequant():
    V, H = 1000, 512
    for qt in (GGMLType.Q4_K, GGMLType.Q8_0):
        w, wd = _qw(V, H, qt, 9)
        ids = torch.tensor([0, 5, 999, 5], dtype=torch.int32, device=DEV)
        out = torch.zeros(4, H, device=DEV)
        ops.embed(w, ids, out_f32=out)
        torch.testing.assert_close(out.cpu(), wd[ids.cpu().long()], rtol=1e-5, atol=1e-6)
        bf = w.dequantize_bf16()
        torch.testing.assert_close(bf.float().cpu(), wd, rtol=1e-2, atol=1e-4)


@pytest.mark.parametrize("act,up", [(0, True), (1, True), (1, False)])
@pytest.mark.parametrize("F", [688, 1024])
def test_swiglu_kernel_matches_fp32(act, up, F):
    """Gated activation kernel (SiLU / GELU-tanh gate, or ungated GELU) against fp32 PyTorch;
    F = 1024 takes the 8-wide vector path, 688 the scalar one."""
    import torch.nn.functional as Fn
    T = 37
    g = torch.Generator().manual_seed(F + act)
    gu = torch.randn(T, 2 * F, generator=g).bfloat16()
    out = torch.zeros(T, F, dtype=torch.bfloat16, device=DEV)
    ops.swiglu(gu.to(DEV), T, F, out_bf16=out, ld_out=F, up_off=F if up else -1, act=act)
    a = gu[:, :F].float()
    gate = Fn.silu(a) if act == 0 else Fn.gelu(a, approximate="tanh")
    ref = gate * (gu[:, F:].float() if up else 1.0)
    torch.testing.assert_close(out.float().cpu(), ref, rtol=1e-2, atol=1e-2)
