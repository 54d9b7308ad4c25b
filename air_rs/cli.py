"""``air-rs`` command line (same subcommands, flags and defaults as the reference's
``src/bin/air_rs.rs:107-360``): ``generate``, ``serve``, ``bench``, ``info``, plus the
README-documented ``pull`` / ``--list-models`` / ``--run`` / ``--interactive`` /
``--serve`` shortcuts that the reference binary lacks.

``--tp N`` relaunches the command as N ranks (one process per GPU, NCCL) through
``torch.distributed.run``; rank 0 prints.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

from . import __version__


def _common(p: argparse.ArgumentParser, serve: bool = False):
    p.add_argument("-m", "--model", required=True, help="Path to GGUF model file (or registry alias)")
    p.add_argument("--ctx-size", type=int, default=None, help="Override context length for the KV budget")
    p.add_argument("--resident", action="store_true", help="Keep all weights in HBM (the default on B200)")
    p.add_argument("--stream-weights", action="store_true",
                   help="S.L.I.P.: keep layer weights in pinned host memory and stream them per forward")
    p.add_argument("--tp", type=int, default=1, help="Tensor-parallel GPUs (default: 1)")
    p.add_argument("--gds", action="store_true",
                   help="Read weights with GPUDirect Storage (cuFile) straight into HBM; falls back to "
                        "parallel reads into pinned buffers when cuFile is unavailable")
    p.add_argument("--enable-auto-tool-choice", action="store_true")
    p.add_argument("--tool-call-parser", default=None,
                   help="llama3_json | hermes | mistral | deepseekv3")
    p.add_argument("--reasoning-format", default="auto" if serve else None, help="none | deepseek | auto")
    p.add_argument("--guided-decoding-backend", default="xgrammar" if serve else None,
                   help="accepted for compatibility; the built-in GBNF engine is always used")
    p.add_argument("--chat-template", default=None, help="chatml | llama3 | mistral | phi3 | gemma")
    p.add_argument("--enable-prefix-caching", action="store_true")
    p.add_argument("--kv-swap", action="store_true", help="Enable the pinned host KV tier")
    p.add_argument("--kv-swap-block-kb", type=int, default=64)
    p.add_argument("--kv-dtype", default=None, choices=("bf16", "fp8"),
                   help="Paged KV pool precision: bf16 (default) or fp8 (E4M3 + a scale per token and head)")
    p.add_argument("--ternary", "--bitnet", dest="ternary", action="store_true")
    p.add_argument("--ternary-cdsc", action="store_true")
    p.add_argument("--device", default=None, help="cuda | cpu (default: cuda when available)")
    p.add_argument("--expert-slots", type=int, default=None,
                   help="MoE: keep experts in host memory with this many resident in VRAM")
    p.add_argument("--trace", default=None, metavar="FILE",
                   help="Record NVTX ranges and host spans; write a Chrome trace to FILE on exit")


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="air-rs", description=f"air-rs {__version__} — LLM inference engine (B200)")
    ap.add_argument("--version", action="version", version=f"air-rs {__version__}")
    ap.add_argument("--list-models", action="store_true", help="List registered models and exit")
    sub = ap.add_subparsers(dest="cmd")

    g = sub.add_parser("generate", help="Generate text")
    _common(g)
    g.add_argument("-p", "--prompt", required=True)
    g.add_argument("-n", "--max-tokens", type=int, default=512)
    g.add_argument("-t", "--temperature", type=float, default=0.7)
    g.add_argument("--top-p", type=float, default=0.9)
    g.add_argument("--top-k", type=int, default=40)
    g.add_argument("--repetition-penalty", type=float, default=1.1)
    g.add_argument("-s", "--stream", action="store_true", help="Stream tokens as they are generated")
    g.add_argument("--council", action="store_true", help="Speculative council drafting")
    g.add_argument("--epsilon", type=float, default=0.15, help="Council JSD threshold")
    g.add_argument("-md", "--model-draft", default=None, help="Draft GGUF for speculative decoding")
    g.add_argument("--draft-max", type=int, default=5)
    g.add_argument("--grammar", default=None, help="GBNF grammar file or 'json'")
    g.add_argument("--seed", type=int, default=0)

    s = sub.add_parser("serve", help="OpenAI-compatible HTTP server")
    s.add_argument("--dp", type=int, default=1,
                   help="Data-parallel replicas: one full model per GPU (cuda:0..N-1) behind one endpoint")
    _common(s, serve=True)
    s.add_argument("-P", "--port", type=int, default=8080)
    s.add_argument("-H", "--host", default="127.0.0.1")
    s.add_argument("--max-num-seqs", "--max-batch-size", dest="max_num_seqs", type=int, default=64)
    s.add_argument("--tls-cert", default=None)
    s.add_argument("--tls-key", default=None)
    s.add_argument("--api-key", action="append", default=None)
    s.add_argument("--model-name", default=None)
    s.add_argument("--content-safety", action="store_true", help="Screen prompts/outputs with the safety gate")
    s.add_argument("--modelfile", default=None, help="Modelfile with SYSTEM / PARAMETER defaults")

    mc = sub.add_parser("mcp", help="Model Context Protocol server on stdio")
    _common(mc)
    mc.add_argument("--model-name", default=None)

    b = sub.add_parser("bench", help="Throughput benchmark")
    _common(b)
    b.add_argument("-n", "--n-tokens", type=int, default=512)
    b.add_argument("-r", "--runs", type=int, default=3)
    b.add_argument("--batch", type=int, default=1)

    i = sub.add_parser("info", help="Print model metadata")
    i.add_argument("-m", "--model", required=True)

    dr = sub.add_parser("doctor", help="Report GPUs, driver / CUDA / NCCL, native extension and host")
    dr.add_argument("--path", default=".", help="Directory whose free disk space to report")
    pl = sub.add_parser("pull", help="Download a GGUF into the local registry")
    pl.add_argument("repo_id")
    pl.add_argument("filename")
    pl.add_argument("--alias", default=None)
    pl.add_argument("--sha256", default=None)
    return ap


def _maybe_relaunch_tp(args, argv):
    if getattr(args, "tp", 1) > 1 and "WORLD_SIZE" not in os.environ:
        cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={args.tp}",
               "--master-addr=127.0.0.1", "--master-port=29517", "-m", "air_rs"] + argv
        os.execv(sys.executable, cmd)


def _engine(args, max_batch=64):
    from .parallel.tp import init_from_env
    from .runtime.builder import engine_from_gguf
    from .hub import resolve
    tp = None
    if args.tp > 1:
        tp = init_from_env("nccl")
    from .config import EngineConfig
    from .runtime import vram_guard
    path = resolve(args.model)
    ec = EngineConfig.from_env()          # AIR_* overrides of the engine defaults
    vram_guard.set_default_fraction(ec.vram_fraction)
    return engine_from_gguf(path, device=args.device, max_batch=max_batch, max_model_len=args.ctx_size, tp=tp,
                            resident=not getattr(args, "stream_weights", False),
                            expert_slots=getattr(args, "expert_slots", None) or ec.expert_slots,
                            prefix_cache=getattr(args, "enable_prefix_caching", False) or ec.prefix_cache,
                            kv_swap=ec.kv_swap, pressure_control=ec.pressure_control, secure_kv=ec.secure_kv,
                            admission=ec.admission,
                            gds=getattr(args, "gds", False),
                            kv_dtype=getattr(args, "kv_dtype", None) or ec.kv_dtype)


def cmd_generate(args) -> int:
    from .api import Engine, GenerateConfig, GbnfConstraint
    core = _engine(args, max_batch=8)
    eng = Engine(core, GenerateConfig(temperature=args.temperature, top_p=args.top_p, top_k=args.top_k,
                                      repetition_penalty=args.repetition_penalty))
    rank0 = int(os.environ.get("RANK", "0")) == 0
    if args.grammar:
        spec = GbnfConstraint.json_mode() if args.grammar == "json" else GbnfConstraint.from_grammar(
            open(args.grammar).read())
        eng.set_grammar(spec)
    cfg = GenerateConfig(max_tokens=args.max_tokens, temperature=args.temperature, top_p=args.top_p,
                         top_k=args.top_k, repetition_penalty=args.repetition_penalty)
    if (args.model_draft or args.council or args.ternary_cdsc) and core.runner is not None:
        from .spec.speculative import SpeculativeDecoder
        draft = (_engine(argparse.Namespace(**{**vars(args), "model": args.model_draft}), max_batch=8)
                 if args.model_draft else None)
        if draft is None and (args.ternary_cdsc or args.ternary):
            # self-drafting: the target's own weights, ternarised
            from .hub import resolve
            from .spec.ternary_draft import ternary_draft_engine
            draft = ternary_draft_engine(resolve(args.model), device=str(core.runner.device))
        if args.council:
            from .spec.medusa import CouncilDecoder
            # voters: the draft model (when given) and the target itself; a draft chain grows
            # only while their next-token distributions agree within epsilon (JSD)
            sd = CouncilDecoder(core, [v for v in (draft, core) if v is not None], epsilon=args.epsilon,
                                k=args.draft_max)
        else:
            sd = SpeculativeDecoder(core, draft, k=args.draft_max)
        ids, stats = sd.generate(core.tokenizer.encode(args.prompt), args.max_tokens, temperature=args.temperature)
        text = core.tokenizer.decode(ids)
        if rank0:
            print(text)
            print(f"[speculative] {stats}", file=sys.stderr)
        return 0
    if args.stream:
        for tok in eng.stream_to_list(args.prompt, cfg) if not rank0 else _iter_stream(eng, args.prompt, cfg):
            if rank0:
                print(tok, end="", flush=True)
        if rank0:
            print()
    else:
        out = eng.generate(args.prompt, cfg)
        if rank0:
            print(out)
    if rank0:
        m = eng.metrics()
        print(f"\n[metrics] TTFT {m.time_to_first_token_ms:.1f} ms | {m.generated_tokens} tokens | "
              f"{m.tokens_per_second:.1f} tok/s", file=sys.stderr)
    return 0


def _iter_stream(eng, prompt, cfg):
    ch = eng._stream_channel(prompt, cfg)
    yield from ch


def cmd_serve(args) -> int:
    if bool(args.tls_cert) != bool(args.tls_key):
        print("error: --tls-cert and --tls-key must be given together", file=sys.stderr)
        return 2
    import uvicorn
    from .serve.app import create_app
    from .serve.dispatcher import EngineDispatcher
    if getattr(args, "dp", 1) > 1 and args.device is None:
        args.device = "cuda:0"
    core = _engine(args, max_batch=args.max_num_seqs)
    name = args.model_name or os.path.splitext(os.path.basename(args.model))[0]
    if args.tp > 1:
        # one HTTP front end on rank 0; the other ranks mirror its engine loop (one port)
        import torch.distributed as dist
        from .serve.distributed import DistributedDispatcher
        ctl = dist.new_group(backend="gloo")
        d = DistributedDispatcher(core, name, group=ctl)
        if d.rank != 0:
            d.serve_follower()
            return 0
    elif getattr(args, "dp", 1) > 1:
        # data-parallel replicas: one engine per GPU, least-in-flight routing
        from .serve.replicas import ReplicaRouter
        reps = [EngineDispatcher(core, name)]
        for i in range(1, args.dp):
            reps.append(EngineDispatcher(_engine(argparse.Namespace(**{**vars(args), "device": f"cuda:{i}"}),
                                                 max_batch=args.max_num_seqs), name))
        d = ReplicaRouter(reps, name)
    else:
        d = EngineDispatcher(core, name)
    safety = None
    if args.content_safety:
        from .safety import ContentSafetyGate
        safety = ContentSafetyGate()
    mf = None
    if args.modelfile:
        from .modelfile import Modelfile
        mf = Modelfile.load(args.modelfile)
    keys = args.api_key or [k for k in os.environ.get("AIR_API_KEYS", "").split(",") if k] or None
    app = create_app(d, name, api_keys=keys, chat_format=args.chat_template,
                     reasoning_format=args.reasoning_format, tool_call_parser=args.tool_call_parser,
                     safety=safety, modelfile=mf)
    try:
        uvicorn.run(app, host=args.host, port=args.port, ssl_certfile=args.tls_cert, ssl_keyfile=args.tls_key,
                    log_level="info")
    finally:
        d.shutdown()          # under --tp this also releases the follower ranks
    return 0


def cmd_mcp(args) -> int:
    from .serve.mcp import McpServer
    core = _engine(args, max_batch=8)
    srv = McpServer()
    name = args.model_name or os.path.splitext(os.path.basename(args.model))[0]
    srv.register_builtin_tools(core.tokenizer, core, name)
    srv.serve_stdio()
    return 0


def cmd_bench(args) -> int:
    import torch
    from .runtime.engine import SamplingParams
    core = _engine(args, max_batch=max(1, args.batch))
    rank0 = int(os.environ.get("RANK", "0")) == 0
    prompt = core.tokenizer.encode("The quick brown fox")
    results = []
    for run in range(args.runs):
        t0 = time.perf_counter()
        rids = [core.add_request(prompt, SamplingParams(max_tokens=args.n_tokens, temperature=0.0, ignore_eos=True))
                for _ in range(args.batch)]
        first = None
        while core.has_unfinished():
            core.step()
            if first is None and any(core.finished.get(r) or True for r in rids):
                first = time.perf_counter()
        if torch.cuda.is_available():
            torch.cuda.synchronize()
        t1 = time.perf_counter()
        n = sum(len(core.finished.pop(r).output_ids) for r in rids)
        results.append({"run": run, "tokens": n, "wall_s": t1 - t0, "tok_s": n / (t1 - t0),
                        "decode_tok_s": (n - args.batch) / max(1e-9, t1 - first), "ttft_ms": (first - t0) * 1e3})
    if rank0:
        for r in results:
            print(json.dumps(r))
        best = max(r["tok_s"] for r in results)
        print(f"air-rs bench: {args.n_tokens} tokens x {args.runs} runs, batch {args.batch}: best {best:.1f} tok/s")
    return 0


def cmd_info(args) -> int:
    from .gguf import read_gguf
    from .models.config import ModelConfig
    g = read_gguf(args.model)
    cfg = ModelConfig.from_gguf_metadata(g.metadata)
    counts = {}
    total = 0
    for t in g.tensors.values():
        counts[t.qtype.name] = counts.get(t.qtype.name, 0) + 1
        total += t.nbytes
    print(f"file:        {args.model}")
    print(f"gguf:        v{g.version}, {len(g.tensors)} tensors, {total / 2**30:.2f} GiB of weights")
    print(f"arch:        {cfg.arch} ({cfg.variant.value}), ffn {cfg.ffn_type.value}, norm {cfg.norm_type.value}")
    print(f"shape:       {cfg.n_layers} layers, hidden {cfg.hidden_dim}, heads {cfg.n_heads}/{cfg.n_kv_heads} "
          f"(d={cfg.head_dim}), ffn {cfg.intermediate_dim}, vocab {cfg.vocab_size}")
    print(f"rope theta:  {cfg.rope_theta}, ctx {cfg.context_length}, eps {cfg.rms_norm_eps}")
    if cfg.n_experts:
        print(f"experts:     {cfg.n_experts} (top-{cfg.moe_top_k})")
    print("types:       " + ", ".join(f"{k}x{v}" for k, v in sorted(counts.items())))
    return 0


def cmd_doctor(args) -> int:
    from .utils.backend import detect
    print(detect(args.path).summary())
    return 0


def main(argv: list[str] | None = None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    # README shortcuts: --run <model> "prompt" / --serve <model> / --interactive <model>
    if argv and argv[0] == "--run" and len(argv) >= 3:
        argv = ["generate", "-m", argv[1], "-p", argv[2], "--stream"] + argv[3:]
    elif argv and argv[0] == "--serve" and len(argv) >= 2:
        argv = ["serve", "-m", argv[1]] + argv[2:]
    elif argv and argv[0] == "--interactive" and len(argv) >= 2:
        from .tui import repl
        return repl(argv[1])
    args = build_parser().parse_args(argv)
    if args.list_models:
        from .hub import ModelRegistry
        for e in ModelRegistry.load().list():
            print(f"{e.alias or '-':16s} {e.repo_id}/{e.filename}  {e.local_path}")
        return 0
    if args.cmd is None:
        build_parser().print_help()
        return 1
    _maybe_relaunch_tp(args, argv)
    if getattr(args, "trace", None):
        from .utils import trace
        trace.enable(True)
        try:
            return _dispatch(args)
        finally:
            trace.dump_chrome(args.trace)
    return _dispatch(args)


def _dispatch(args) -> int:
    if args.cmd == "pull":
        from .hub import pull
        print(pull(args.repo_id, args.filename, args.alias, args.sha256))
        return 0
    return {"generate": cmd_generate, "serve": cmd_serve, "bench": cmd_bench, "info": cmd_info,
            "mcp": cmd_mcp, "doctor": cmd_doctor}[args.cmd](args)


if __name__ == "__main__":
    sys.exit(main())
