"""Fused tensor-parallel all-reduce kernels (peer push + reduce-RMSNorm-quant).

Ranks are emulated on one GPU with ``PeerComm.local_group``: every rank's receive buffer is
a local allocation, the producers (which never wait) run before the consumers, and all
ranks' consumers run as CTAs of one launch (``reduce_norm_group``), so no launch ever waits
on another launch. Both data paths are covered: one-shot (every partial to every rank) and
two-shot (reduce-scatter to the column owners, then all-gather of the reduced values)."""
import pytest
import torch

from air_rs import ops
from air_rs.gguf import GGMLType, quantize
from air_rs.parallel.symm import PeerComm

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _norm_ref(x, w, eps=1e-5):
    return x / torch.sqrt((x * x).mean(-1, keepdim=True) + eps) * w


def _consume(comms, xs, w, B, K):
    outs = []
    for _ in comms:
        outs.append((torch.zeros(B, K, dtype=torch.int8, device=DEV),
                     torch.zeros(B, K // 32, 2, dtype=torch.float32, device=DEV),
                     torch.zeros(B, K, dtype=torch.bfloat16, device=DEV)))
    PeerComm.reduce_norm_group(comms, xs, w, 1e-5, [o[0] for o in outs], [o[1] for o in outs],
                               [o[2] for o in outs], B)
    return outs


@pytest.mark.parametrize("world,B,K", [(2, 5, 1024), (4, 5, 1024), (8, 5, 1024),
                                       (4, 12, 1024), (8, 16, 4096), (8, 10, 1056), (3, 9, 2048)])
def test_push_reduce_rounds(world, B, K):
    comms = PeerComm.local_group(world, max_rows=16, hidden=K, device=DEV)
    assert comms[0].two_shot(B) == (world > 2 and B >= 9)
    g = torch.Generator().manual_seed(world)
    w = (torch.rand(K, generator=g) + 0.5).to(DEV)
    x0 = torch.randn(B, K, generator=g).to(DEV)
    xs = [x0.clone() for _ in range(world)]
    ref = x0.clone()
    for rnd in range(3):                                   # both parities, epoch advance
        parts = [torch.randn(B, K, generator=g).to(DEV) for _ in range(world)]
        for c, p in zip(comms, parts):
            c.push(p, B)
        outs = _consume(comms, xs, w, B, K)
        ref = ref + sum(parts)
        for x, (xq, xds, y) in zip(xs, outs):
            torch.testing.assert_close(x, ref, rtol=1e-5, atol=1e-5)
            yr = _norm_ref(ref, w)
            torch.testing.assert_close(y.float(), yr, rtol=1e-2, atol=1e-2)
            deq = (xq.float().reshape(B, -1, 32) * xds[..., 0:1]).reshape(B, K)
            torch.testing.assert_close(deq, yr, rtol=0, atol=float(yr.abs().max()) / 120)
    for c in comms:
        c.check()
        assert int(c.epoch.item()) == 3


@pytest.mark.parametrize("world,two_shot", [(2, False), (4, True), (8, True)])
def test_gemv_epilogue_push_matches_store(world, two_shot):
    """Row-parallel Q4_K GEMV with the push epilogue == per-rank partials summed."""
    B, H, Kr = 3, 512, 1024
    comms = PeerComm.local_group(world, max_rows=8, hidden=H, device=DEV)
    for c in comms:
        c.two_shot_min_rows = 1 if two_shot else 1000
    assert comms[0].two_shot(B) == two_shot
    g = torch.Generator().manual_seed(0)
    ws = [ops.QWeight.from_raw(quantize(torch.randn(H, Kr, generator=g) * 0.02, GGMLType.Q4_K),
                               GGMLType.Q4_K, H, Kr, DEV) for _ in range(world)]
    acts = [torch.randn(B, Kr, generator=g).to(DEV) for _ in range(world)]
    x0 = torch.randn(B, H, generator=g).to(DEV)
    ref = x0.clone()
    qs = []
    for a in acts:
        xq = torch.empty(B, Kr, dtype=torch.int8, device=DEV)
        xds = torch.empty(B, Kr // 32, 2, dtype=torch.float32, device=DEV)
        ops.rmsnorm_quant(a, None, 0.0, xq, xds)
        qs.append((xq, xds))
    for w, (xq, xds) in zip(ws, qs):
        out = torch.zeros(B, H, device=DEV)
        ops.gemv(w, xq, xds, B, ops.EPI_STORE, out_f32=out)
        ref += out
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    for c, w, (xq, xds) in zip(comms, ws, qs):
        c.push_gemv(w, xq, xds, B, err=err)
    xs = [x0.clone() for _ in range(world)]
    wn = torch.ones(H, device=DEV)
    _consume(comms, xs, wn, B, H)
    for x in xs:
        torch.testing.assert_close(x, ref, rtol=1e-4, atol=1e-4)
    assert int(err.item()) == 0


def test_reduce_wait_times_out_without_producer():
    """A flag that nothing sets: the bounded wait gives up, reports code 2, and the
    context stays usable."""
    B, K = 2, 256
    (c0, c1) = PeerComm.local_group(2, max_rows=4, hidden=K, device=DEV, timeout_s=0.05)
    c0.push(torch.ones(B, K, device=DEV), B)           # rank 1 never pushes
    x = torch.zeros(B, K, device=DEV)
    c0.reduce_norm(x, torch.ones(K, device=DEV), 1e-5, None, None, None, B)
    torch.cuda.synchronize()
    assert int(c0.err.item()) == 2
    with pytest.raises(RuntimeError):
        c0.check()
    assert float((torch.ones(4, device=DEV) * 2).sum()) == 8.0


def test_graph_replay_advances_epochs():
    world, B, K = 2, 4, 512
    comms = PeerComm.local_group(world, max_rows=B, hidden=K, device=DEV)
    parts = [torch.randn(B, K, device=DEV) for _ in range(world)]
    xs = [torch.zeros(B, K, device=DEV) for _ in range(world)]
    w = torch.ones(K, device=DEV)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for c, p in zip(comms, parts):
                c.push(p, B)
            PeerComm.reduce_norm_group(comms, xs, w, 1e-5, B=B)
    torch.cuda.current_stream().wait_stream(s)
    for x in xs:
        x.zero_()
    for _ in range(5):
        g.replay()
    torch.cuda.synchronize()
    total = sum(parts)
    for c, x in zip(comms, xs):
        torch.testing.assert_close(x, 5 * total, rtol=1e-5, atol=1e-4)
        assert int(c.epoch.item()) == 5
        c.check()


@pytest.mark.parametrize("world,T", [(2, 24), (4, 32), (8, 16)])   # T x world <= 148 (one launch)
def test_gemm_epilogue_push_matches_store(world, T):
    """Row-parallel tcgen05 GEMM (Q4_K) whose epilogue pushes into the peer buffers: the
    reduced residual equals the sum of the per-rank GEMM outputs (fp32 reference of the
    same products, computed with the store epilogue)."""
    from air_rs.ops import gemm
    H, Kr = 1024, 2048
    comms = PeerComm.local_group(world, max_rows=T, hidden=H, device=DEV)
    g = torch.Generator().manual_seed(world)
    ws = [ops.QWeight.from_raw(quantize(torch.randn(H, Kr, generator=g) * 0.02, GGMLType.Q4_K),
                               GGMLType.Q4_K, H, Kr, DEV) for _ in range(world)]
    acts = [(torch.randn(T, Kr, generator=g)).to(DEV, torch.bfloat16) for _ in range(world)]
    x0 = torch.randn(T, H, generator=g).to(DEV)
    ref = x0.clone()
    for w, a in zip(ws, acts):
        out = torch.zeros(T, H, device=DEV)
        gemm.linear(a, w, out)
        ref += out
        # the store epilogue agrees with an fp32 PyTorch product of the dequantised weight
        r32 = a.float() @ w.dequantize_bf16().float().t()
        # A is rounded to bf16 after the GGUF scale math (same bound as the GEMM tests)
        torch.testing.assert_close(out, r32, rtol=2e-2, atol=1e-2 * float(r32.abs().max()))
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    dummy = torch.zeros(T, H, device=DEV)
    for c, w, a in zip(comms, ws, acts):
        c.push_gemm(a, w, dummy, err=err)
    xs = [x0.clone() for _ in range(world)]
    _consume(comms, xs, torch.ones(H, device=DEV), T, H)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    for c, x in zip(comms, xs):
        c.check()
        torch.testing.assert_close(x, ref, rtol=1e-4, atol=1e-4)
