"""tcgen05 dequant-fused GEMM vs a plain PyTorch fp32 reference."""
import pytest
import torch

from air_rs import ops
from air_rs.gguf import GGMLType, quantize, dequantize
from air_rs.ops import gemm

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _w(N, K, qt, seed):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(N, K, generator=g) * 0.02
    raw = quantize(w, qt)
    wd = dequantize(raw, qt).reshape(N, K)
    return ops.QWeight.from_raw(raw, qt, N, K, DEV), wd


@pytest.mark.parametrize("qt", [GGMLType.Q4_K, GGMLType.Q8_0, GGMLType.FP8_E4M3_B128, GGMLType.BF16])
@pytest.mark.parametrize("N,K,T,splits", [(128, 256, 1, 1), (384, 512, 5, 1), (256, 1024, 64, None),
                                          (256, 2048, 64, 4), (512, 1024, 200, None), (4096, 4096, 16, None),
                                          (200, 512, 33, None), (1456, 256, 33, 1),
                                          (1024, 2048, 512, None), (384, 1024, 300, 3),
                                          (256, 512, 129, 1)])     # 256-token tiles
def test_gemm_q_store(qt, N, K, T, splits):
    w, wd = _w(N, K, qt, 1)
    assert gemm.tc_supported(w)          # the tcgen05 kernel, not the library fallback
    g = torch.Generator().manual_seed(2)
    x = torch.randn(T, K, generator=g).bfloat16()
    ref = x.float() @ wd.bfloat16().float().t()
    out = torch.zeros(T, N, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    gemm.linear(x.to(DEV), w, out, splits=splits, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    tol = 1e-2 * float(ref.abs().max())  # A is rounded to bf16 after the GGUF scale math
    torch.testing.assert_close(out.cpu(), ref, rtol=2e-2, atol=tol)
    outb = torch.zeros(T, N, dtype=torch.bfloat16, device=DEV)
    gemm.linear(x.to(DEV), w, outb, splits=splits)
    torch.testing.assert_close(outb.float().cpu(), ref, rtol=2e-2, atol=2 * tol)


def test_gemm_q_residual_and_repeat():
    N, K, T = 512, 4096, 64
    w, wd = _w(N, K, GGMLType.Q4_K, 3)
    x = (torch.randn(T, K) * 0.5).bfloat16()
    ref = x.float() @ wd.bfloat16().float().t()
    resid = torch.ones(T, N, device=DEV)
    for i in range(3):  # the split-K counters must reset themselves between calls
        gemm.linear(x.to(DEV), w, resid, residual=True)
    torch.testing.assert_close(resid.cpu(), 1 + 3 * ref, rtol=2e-2, atol=3e-2 * float(ref.abs().max()))


@pytest.mark.parametrize("T,rot,bias", [(40, 128, False), (300, 128, True), (17, 64, False)])
def test_gemm_qkv_rope_epilogue_matches_separate_kernel(T, rot, bias):
    """QKV GEMM whose epilogue adds the bias, applies RoPE and writes q and the paged K/V,
    against the same GEMM storing bf16 followed by the token-parallel RoPE/KV kernel."""
    nh, nkv, hd, bs = 4, 2, 128, 16
    N, K = (nh + 2 * nkv) * hd, 512
    w, _ = _w(N, K, GGMLType.Q4_K, 7)
    g = torch.Generator().manual_seed(T)
    x = torch.randn(T, K, generator=g).bfloat16().to(DEV)
    cs = ops.rope_table(1024, rot, 10000.0, DEV)
    pos = torch.randint(0, 1000, (T,), generator=g, dtype=torch.int32).to(DEV)
    nblk = (T + bs - 1) // bs + 2
    slots = torch.randperm(nblk * bs, generator=g)[:T].to(torch.int64)
    slots[::7] = -1                                              # rows without a cache slot
    slots = slots.to(DEV)
    b = (torch.randn(N, generator=g) * 0.1).to(DEV) if bias else None
    kv_a = torch.zeros(nblk, 2, nkv, bs, hd, dtype=torch.bfloat16, device=DEV)
    kv_b = torch.zeros_like(kv_a)
    q_a = torch.zeros(T, nh, hd, device=DEV)
    q_b = torch.zeros_like(q_a)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    qkv = torch.zeros(T, N, dtype=torch.bfloat16, device=DEV)
    gemm.linear(x, w, qkv, err=err, rope=dict(cs=cs, positions=pos, slots=slots, kv=kv_a, q_out=q_a, bias=b,
                                               n_heads=nh, n_kv=nkv, block_size=bs, rot_dim=rot))
    gemm.linear(x, w, qkv, err=err)
    ops.rope_kv(qkv, T, cs, pos, slots, kv_b, q_b, n_heads=nh, n_kv=nkv, head_dim=hd, block_size=bs,
                rot_dim=rot, err=err, bias=b)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    scale = float(q_b.abs().max())
    torch.testing.assert_close(q_a, q_b, rtol=2e-2, atol=1e-2 * scale)
    torch.testing.assert_close(kv_a.float(), kv_b.float(), rtol=2e-2, atol=1e-2 * scale)
