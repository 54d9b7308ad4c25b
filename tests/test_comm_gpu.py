"""Fused tensor-parallel all-reduce kernels (peer push + reduce-RMSNorm-quant).

Ranks are emulated on one GPU with ``PeerComm.local_group``: every rank's receive buffer is
a local allocation, and the producers (which never wait) run before the consumers, so no
launch ever waits on another launch that has not finished."""
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
    for c, x in zip(comms, xs):
        xq = torch.zeros(B, K, dtype=torch.int8, device=DEV)
        xds = torch.zeros(B, K // 32, 2, dtype=torch.float32, device=DEV)
        y = torch.zeros(B, K, dtype=torch.bfloat16, device=DEV)
        c.reduce_norm(x, w, 1e-5, xq, xds, y, B)
        outs.append((xq, xds, y))
    return outs


@pytest.mark.parametrize("world", [2, 4, 8])
def test_push_reduce_rounds(world):
    B, K = 5, 1024
    comms = PeerComm.local_group(world, max_rows=8, hidden=K, device=DEV)
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


def test_gemv_epilogue_push_matches_store():
    """Row-parallel Q4_K GEMV with the push epilogue == per-rank partials summed."""
    world, B, H, Kr = 2, 3, 512, 1024
    comms = PeerComm.local_group(world, max_rows=8, hidden=H, device=DEV)
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
            for c, x in zip(comms, xs):
                c.reduce_norm(x, w, 1e-5, None, None, None, B)
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
