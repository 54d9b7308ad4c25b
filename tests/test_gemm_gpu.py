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
def test_gemm_q_store(qt, N, K, T, splits, monkeypatch):
    monkeypatch.setenv("AIR_FP8_MMA", "0")   # FP8: the dequantising path (W8A8 has its own tests)
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
