"""Per-kernel microbenchmarks at Llama-3-8B decode / prefill shapes.

``--op graph`` measures CUDA-graph launch overhead: one decode step of a random-init model
(``--preset``, default llama3-8b) at batch B run eagerly (every kernel launched from Python)
and as a replayed graph, device time per step from CUDA events plus host time per step, and
the number of kernels in the step.

``--op prefill`` lists the kernels of one ``--batch``-token prefill (default 512) the same
way, then its CUDA-event time (the device part of TTFT).

``--op step`` lists the kernels of one graph-replayed decode step (CUPTI through
``torch.profiler``: count and device time per kernel over 10 steps) at ``--batch`` rows of
``--ctx`` context tokens, then the CUDA-event time per step.

``python -m air_rs.perf.microbench [--op gemv|gemm|attn|norm|graph|step|all] [--name qkv|o|gateup|down|lm]
[--batch B] [--iters N]`` prints one line per case: device time (CUDA events around a CUDA
graph of N back-to-back launches, after warm-up), achieved bytes/s or FLOP/s, and the
fraction of the measured HBM copy bandwidth / cuBLAS bf16 rate (``MEASURED_PEAKS.json`` at
the repo root when present, else 6.65 TB/s and 1.59 PFLOP/s). Weights rotate over enough
copies that every launch streams from HBM (working set > L2).
"""
from __future__ import annotations

import argparse
import json
import os

import torch

from .. import ops
from ..gguf import GGMLType

SHAPES = {"qkv": (6144, 4096), "o": (4096, 4096), "gateup": (28672, 4096), "down": (4096, 14336),
          "lm": (128256, 4096)}


def tp_shapes(tp: int) -> dict:
    """One rank's shard of each projection under tensor parallelism: QKV / gate|up / LM head
    split by output rows, O / down by input columns."""
    return {"qkv": (6144 // tp, 4096), "o": (4096, 4096 // tp), "gateup": (28672 // tp, 4096),
            "down": (4096, 14336 // tp), "lm": (128256 // tp, 4096)}
L2_BYTES = 126e6


def peaks() -> tuple[float, float, str]:
    p = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return d["hbm_gbs"] * 1e9, d["bf16_tflops"] * 1e12, "of measured"
    except (OSError, KeyError, ValueError):
        return 6.65e12, 1.59e15, "of fallback"


def ev_time(fn, iters: int = 20) -> float:
    """Mean microseconds per call over a graph of ``iters`` calls."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for _ in range(iters):
                fn()
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    g.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters * 1e3


def _q4k_weights(N: int, K: int, dev, min_bytes: float = 4 * L2_BYTES):
    """Random Q4_K tiles (valid f16 d/dmin) in enough copies to exceed L2."""
    nb = K // 256
    one = N * nb * 144
    copies = max(1, int(min_bytes // one) + 1)
    ws = []
    for _ in range(copies):
        d = torch.randint(0, 255, (N // 128, nb, 128, 144), dtype=torch.uint8, device=dev)
        d[..., 0:4] = torch.tensor([0, 0x20, 0, 0x20], dtype=torch.uint8, device=dev)   # d = dmin = 2^-7
        ws.append(ops.QWeight(ops.FMT_Q4K, d, None, N, K, GGMLType.Q4_K))
    return ws, one


def bench_gemv(name: str, B: int, iters: int, dev):
    N, K = SHAPES[name]
    ws, nbytes = _q4k_weights(N, K, dev)
    xq = torch.randint(-100, 100, (B, K), dtype=torch.int8, device=dev)
    xds = torch.rand(B, K // 32, 2, device=dev)
    out = torch.zeros(B, N, device=dev)
    i = [0]

    def f():
        w = ws[i[0] % len(ws)]
        i[0] += 1
        if name == "gateup":
            ops.gemv(w.rows(0, N // 2), xq, xds, B, ops.EPI_SWIGLU, w2=w.rows(N // 2, N), out_f32=out, ld_out=N)
        else:
            ops.gemv(w, xq, xds, B, ops.EPI_STORE, out_f32=out)
    us = ev_time(f, iters)
    return us, nbytes, 2.0 * N * K * B


def _fp8_weights(N: int, K: int, dev, min_bytes: float = 4 * L2_BYTES):
    """Random block-scaled FP8 weights (E4M3 codes + f32 multiplier per 128-wide block)."""
    one = N * K + N * (K // 128) * 4
    copies = max(1, int(min_bytes // one) + 1)
    ws = []
    for _ in range(copies):
        codes = torch.randn(N, K, device=dev).to(torch.float8_e4m3fn).view(torch.uint8)
        sc = torch.rand(N, K // 128, device=dev) * 0.01
        ws.append(ops.QWeight(ops.FMT_FP8, codes, sc, N, K, GGMLType.FP8_E4M3_B128))
    return ws, one


def bench_gemm(name: str, T: int, iters: int, dev, wfmt: str = "q4k"):
    """wfmt: q4k (dequant-fused GEMM), fp8 (FP8 codes dequantised to bf16 in the GEMM), fp8mma
    (W8A8: activation quantisation + the kind::f8f6f4 kernel)."""
    from ..ops import gemm
    N, K = SHAPES[name]
    ws, nbytes = _q4k_weights(N, K, dev) if wfmt == "q4k" else _fp8_weights(N, K, dev)
    x = torch.randn(T, K, device=dev).bfloat16()
    out = torch.zeros(T, N, device=dev, dtype=torch.bfloat16)
    i = [0]

    def f():
        if wfmt == "fp8mma":
            gemm.linear_fp8(x, ws[i[0] % len(ws)], out)
        else:
            gemm.linear(x, ws[i[0] % len(ws)], out)
        i[0] += 1
    us = ev_time(f, iters)
    return us, nbytes + T * K * 2 + T * N * 2, 2.0 * N * K * T


def bench_attn(B: int, ctx: int, iters: int, dev, tp: int = 1, kv_dtype: str = "bf16"):
    nkv, nh, d, bs = 8 // tp, 32 // tp, 128, 16
    nblk = B * ((ctx + bs - 1) // bs)
    row = d * 2 if kv_dtype == "bf16" else d + 16
    copies = max(1, int(4 * L2_BYTES // (nblk * 2 * nkv * bs * row)) + 1)
    if kv_dtype == "fp8":
        from ..kv.fp8 import quantize_rows
        kvs = [quantize_rows(torch.randn(nblk, 2, nkv, bs, d, device=dev)) for _ in range(copies)]
    else:
        kvs = [torch.randn(nblk, 2, nkv, bs, d, device=dev).bfloat16() for _ in range(copies)]
    bt = torch.arange(nblk, dtype=torch.int32, device=dev).view(B, -1)
    q = torch.randn(B, nh, d, device=dev)
    out = torch.zeros(B, nh, d, device=dev)
    ns = max(1, min(32, -(-4 * 148 // (B * nkv))))
    po = torch.zeros(B * nh * ns * d, device=dev)
    pm = torch.zeros(B * nh * ns * 2, device=dev)
    cl = torch.full((B,), ctx, dtype=torch.int32, device=dev)
    i = [0]

    def f():
        ops.paged_attention(q, kvs[i[0] % copies], bt, cl, out, n_rows=B, n_heads=nh, n_kv=nkv, head_dim=d,
                            block_size=bs, n_splits=ns, split_tokens=0, part_o=po, part_ml=pm)
        i[0] += 1
    us = ev_time(f, iters)
    return us, B * ctx * 2 * nkv * row, 4.0 * B * nh * ctx * d


def bench_graph(preset: str, B: int, iters: int, dev) -> dict:
    """Eager vs graph-replayed decode step of a random-init model at batch ``B``."""
    import time
    from ..runtime.builder import random_engine
    eng = random_engine(preset, device=dev, max_batch=max(B, 1), max_model_len=1024, num_blocks=B * 64 + 16)
    rn = eng.runner
    prompts = [[(7 * i + j) % 200 + 3 for j in range(32)] for i in range(B)]
    from ..runtime.engine import SamplingParams
    for p in prompts:
        eng.add_request(p, SamplingParams(max_tokens=900, temperature=0.0, ignore_eos=True))
    eng.step()                       # prefill + first decode step
    bucket = eng._bucket(B)
    out = {"preset": preset, "B": B, "bucket": bucket}
    for mode in ("eager", "graph"):
        use_graph = mode == "graph"
        for _ in range(3):
            rn.decode(bucket, use_graph=use_graph)
        torch.cuda.synchronize()
        c0 = ops.launch_count()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        a.record()
        for _ in range(iters):
            rn.decode(bucket, use_graph=use_graph)
        b.record()
        host = (time.perf_counter() - t0) / iters * 1e3
        torch.cuda.synchronize()
        out[mode] = {"device_ms": a.elapsed_time(b) / iters, "host_ms": host,
                     "kernels": (ops.launch_count() - c0) // iters}
    out["graph_speedup"] = out["eager"]["device_ms"] / out["graph"]["device_ms"]
    for r in list(eng.running):
        eng.abort(r.rid)
    return out


def profile_step(preset: str, B: int, ctx: int, dev) -> str:
    from torch.profiler import ProfilerActivity, profile
    from ..runtime.builder import random_engine
    from ..runtime.engine import SamplingParams
    eng = random_engine(preset, device=dev, max_batch=max(B, 1), max_model_len=ctx + 1024,
                        num_blocks=B * ((ctx + 1024) // 16 + 2) + 16)
    for i in range(B):
        eng.add_request([(7 * i + j) % 200 + 3 for j in range(ctx)],
                        SamplingParams(max_tokens=900, temperature=0.0, ignore_eos=True))
    eng.step()
    rn, bucket = eng.runner, eng._bucket(B)
    for _ in range(5):
        rn.decode(bucket)
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(10):
            rn.decode(bucket)
        torch.cuda.synchronize()
    table = prof.key_averages().table(sort_by="cuda_time_total", row_limit=20, max_name_column_width=80)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(20):
        rn.decode(bucket)
    b.record()
    torch.cuda.synchronize()
    for r in list(eng.running):
        eng.abort(r.rid)
    return table + f"\n{preset} decode B={B} ctx={ctx}: {a.elapsed_time(b) / 20:.3f} ms/step (CUDA events, graph replay)"


def profile_prefill(preset: str, T: int, dev) -> str:
    """Kernels of one T-token prefill (prompt -> first token): CUPTI through torch.profiler,
    count and device time per kernel over 3 prefills, then the CUDA-event time of one."""
    from torch.profiler import ProfilerActivity, profile
    from ..runtime.builder import random_engine
    from ..runtime.engine import SamplingParams
    eng = random_engine(preset, device=dev, max_batch=8, max_model_len=T + 64, num_blocks=8 * ((T + 64) // 16 + 2))

    def one(i):
        eng.add_request([(7 * i + j) % 200 + 3 for j in range(T)],
                        SamplingParams(max_tokens=1, temperature=0.0, ignore_eos=True))
        eng._prefill(eng._admit())

    for i in range(3):
        one(i)
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for i in range(3):
            one(10 + i)
        torch.cuda.synchronize()
    table = prof.key_averages().table(sort_by="cuda_time_total", row_limit=25, max_name_column_width=80)
    ts = []
    for i in range(5):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        one(20 + i)
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    ts.sort()
    return table + f"\n{preset} prefill T={T}: {ts[len(ts) // 2]:.3f} ms median of 5 (CUDA events)"


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--op", default="all", choices=["all", "gemv", "gemm", "attn", "norm", "graph", "step", "prefill"])
    ap.add_argument("--preset", default="llama3-8b")
    ap.add_argument("--name", default=None, choices=list(SHAPES))
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--ctx", type=int, default=640)
    ap.add_argument("--kv-dtype", default="bf16", choices=["bf16", "fp8"])
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--wfmt", default="q4k", choices=["q4k", "fp8", "fp8mma"], help="GEMM weight format / path")
    ap.add_argument("--tp", type=int, default=1, help="shapes of one rank's shard under tensor parallelism")
    a = ap.parse_args(argv)
    dev = torch.device("cuda")
    if a.tp > 1:
        SHAPES.update(tp_shapes(a.tp))
    bw, fl, tag = peaks()
    names = [a.name] if a.name else list(SHAPES)

    def line(kind, desc, us, nbytes, flops):
        print(f"{kind:5s} {desc:34s} {us:9.1f} us  {nbytes / us / 1e3:7.0f} GB/s ({nbytes / us * 1e6 / bw:5.2f} {tag})"
              f"  {flops / us / 1e6:7.1f} TFLOP/s ({flops / us * 1e6 / fl:5.3f} {tag})", flush=True)

    if a.op in ("all", "gemv"):
        for n in names:
            for B in ([a.batch] if a.batch else [1, 8]):
                us, nb, f = bench_gemv(n, B, a.iters, dev)
                line("gemv", f"{n} N={SHAPES[n][0]} K={SHAPES[n][1]} B={B}", us, nb, f)
    if a.op in ("all", "gemm"):
        for n in names:
            for T in ([a.batch] if a.batch else [16, 64, 512]):
                us, nb, f = bench_gemm(n, T, a.iters, dev, a.wfmt)
                line("gemm", f"{a.wfmt} {n} N={SHAPES[n][0]} K={SHAPES[n][1]} T={T}", us, nb, f)
    if a.op in ("all", "attn"):
        for B in ([a.batch] if a.batch else [1, 64]):
            us, nb, f = bench_attn(B, a.ctx, a.iters, dev, a.tp, a.kv_dtype)
            line("attn", f"decode B={B} ctx={a.ctx} kv={a.kv_dtype}", us, nb, f)
    if a.op in ("all", "norm"):
        for K, B in [(4096, 1), (4096, 64), (14336, 8)]:
            x = torch.randn(B, K, device=dev)
            w = torch.rand(K, device=dev)
            q = torch.empty(B, K, dtype=torch.int8, device=dev)
            ds = torch.empty(B, K // 32, 2, device=dev)
            us = ev_time(lambda: ops.rmsnorm_quant(x, w, 1e-5, q, ds), a.iters)
            line("norm", f"rmsnorm_quant K={K} B={B}", us, B * K * 4 + B * K + B * K // 8, 0.0)

    if a.op == "step":
        print(profile_step(a.preset, a.batch or 1, a.ctx, dev), flush=True)
    if a.op == "prefill":
        print(profile_prefill(a.preset, a.batch or 512, dev), flush=True)
    if a.op == "graph":
        for B in ([a.batch] if a.batch else [1, 64]):
            r = bench_graph(a.preset, B, a.iters, dev)
            e, g = r["eager"], r["graph"]
            print(f"graph {a.preset} decode B={B}: eager {e['device_ms']:.3f} ms/step (host {e['host_ms']:.3f}), "
                  f"graph {g['device_ms']:.3f} ms/step (host {g['host_ms']:.3f}), {g['kernels']} kernels/step, "
                  f"speedup {r['graph_speedup']:.2f}x", flush=True)


if __name__ == "__main__":
    main()
