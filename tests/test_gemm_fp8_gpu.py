"""W8A8 FP8 tcgen05 GEMM (kind::f8f6f4, per-block scale promotion) and its activation
quantiser vs plain PyTorch fp32 restatements of the same ops."""
import pytest
import torch

from air_rs import ops
from air_rs.gguf import GGMLType
from air_rs.ops import gemm

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _fp8_weight(N, K, seed):
    g = torch.Generator().manual_seed(seed)
    codes = (torch.randn(N, K, generator=g) * 2).to(torch.float8_e4m3fn)
    sc = torch.rand(N, K // 128, generator=g) * 0.02 + 0.001
    wd = codes.float() * sc.repeat_interleave(128, dim=1)
    w = ops.QWeight(ops.FMT_FP8, codes.view(torch.uint8).to(DEV), sc.to(DEV), N, K, GGMLType.FP8_E4M3_B128)
    return w, wd


def _quant_ref(x):
    """fp32 restatement of the activation quantiser: per row amax / 448."""
    xf = x.float()
    amax = xf.abs().amax(-1)
    scale = amax / 448.0
    inv = torch.where(amax > 0, 448.0 / amax, torch.zeros_like(amax))
    q = (xf * inv[:, None]).clamp(-448, 448).to(torch.float8_e4m3fn)
    return q, scale


@pytest.mark.parametrize("T,K", [(1, 128), (7, 512), (64, 4096), (300, 256)])
def test_quant_fp8_rows(T, K):
    g = torch.Generator().manual_seed(T + K)
    x = (torch.randn(T, K, generator=g) * 3).bfloat16()
    x[0] = 0                                             # an all-zero row
    xq, xs = gemm.quant_fp8_rows(x.to(DEV))
    torch.cuda.synchronize()
    q_ref, s_ref = _quant_ref(x)
    torch.testing.assert_close(xs.cpu(), s_ref, rtol=1e-6, atol=0)
    # same codes up to a rounding difference of one E4M3 step (relative 1/8) on a few elements
    torch.testing.assert_close(xq.cpu().view(torch.float8_e4m3fn).float(), q_ref.float(), rtol=0.13, atol=2 ** -9)
    assert (xq.cpu() != q_ref.view(torch.uint8)).float().mean() < 0.01


@pytest.mark.parametrize("N,K,T,splits", [(128, 128, 1, 1), (384, 512, 5, 1), (300, 1024, 33, None),
                                          (256, 2048, 64, 4), (4096, 4096, 64, None), (512, 1024, 100, None),
                                          (1456, 512, 200, 2), (28672 // 8, 4096, 16, None),
                                          (28672, 1024, 64, None), (384, 1024, 300, 3), (640, 512, 129, 1)])
def test_gemm_fp8_store(N, K, T, splits):
    w, wd = _fp8_weight(N, K, 1)
    g = torch.Generator().manual_seed(2)
    x = torch.randn(T, K, generator=g).bfloat16()
    xd = x.to(DEV)
    xq, xs = gemm.quant_fp8_rows(xd)
    torch.cuda.synchronize()
    # reference of the same op: the quantised activations (as the kernel saw them) x weights, fp32
    xdq = xq.cpu().view(torch.float8_e4m3fn).float() * xs.cpu()[:, None]
    ref = xdq @ wd.t()
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = torch.zeros(T, N, device=DEV)
    gemm.linear_fp8(xd, w, out, splits=splits, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    scale = float(ref.abs().max())
    torch.testing.assert_close(out.cpu(), ref, rtol=1e-3, atol=1e-4 * scale)
    # against the bf16 activations: only the E4M3 activation rounding differs
    ref_bf = x.float() @ wd.t()
    assert float((out.cpu() - ref_bf).abs().max()) < 0.08 * float(ref_bf.abs().max())
    # bf16 store and residual add
    outb = torch.zeros(T, N, dtype=torch.bfloat16, device=DEV)
    gemm.linear_fp8(xd, w, outb, splits=splits, err=err)
    res = torch.randn(T, N, generator=g).to(DEV)
    res0 = res.clone()
    gemm.linear_fp8(xd, w, res, residual=True, splits=splits, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    torch.testing.assert_close(outb.cpu().float(), ref, rtol=1e-2, atol=1e-2 * scale)
    torch.testing.assert_close((res - res0).cpu(), ref, rtol=1e-3, atol=1e-3 * scale)


def test_linear_dispatch_fp8_mma(monkeypatch):
    """AIR_FP8_MMA=1 sends FP8 weights through the W8A8 kernel from the generic entry point,
    repeatably (split-K counters reset themselves between calls)."""
    monkeypatch.setenv("AIR_FP8_MMA", "1")
    w, wd = _fp8_weight(1024, 2048, 3)
    x = torch.randn(64, 2048).bfloat16().to(DEV)
    outs = []
    for _ in range(3):
        out = torch.zeros(64, 1024, device=DEV)
        gemm.linear(x, w, out)
        outs.append(out)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
    ref = x.float().cpu() @ wd.t()
    assert float((outs[0].cpu() - ref).abs().max()) < 0.08 * float(ref.abs().max())
