"""Model runner: one batched forward over the paged KV pool, on the sm_100a kernels.

``decode(B)`` runs one token for B sequences; its buffers are static per batch bucket so
the whole step (embedding -> layers -> LM head -> sampler) is captured once in a CUDA
graph and replayed (the reference's graph registry ``src/strix/gpu_direct.rs:1054-1113`` is
a stub; this one is real). ``prefill`` runs any number of prompt tokens of one or more
sequences (chunked prefill) through the GEMM path and samples each sequence's next token.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass

import torch

from .. import ops
from ..parallel.tp import COMM
from ..models.config import ModelConfig
from ..models.llama import LlamaWeights
from ..utils import trace

# The int8-activation GEMV chain serves decode batches up to GEMV_LIMIT_B (its buffers are
# sized for that); by default only up to GEMV_MAX_B, above which the tensor-core GEMM step is
# faster (Llama-3-8B Q4_K on B200: B=4 3.63 vs 4.30 ms per step, B=8 3.65 vs 7.88 ms).
# AIR_GEMV_MAX_B overrides; ModelRunner.gemv_max_b per runner.
GEMV_LIMIT_B = 8
GEMV_MAX_B = max(1, min(GEMV_LIMIT_B, int(os.environ.get("AIR_GEMV_MAX_B", "2"))))


def _dev_param(x, dtype, device):
    return torch.tensor(x, dtype=dtype, device=device)


@dataclass
class StepInputs:
    """Static per-bucket device inputs of one decode step."""
    ids: torch.Tensor          # [B] int32 (written by the previous step's sampler)
    positions: torch.Tensor    # [B] int32
    slots: torch.Tensor        # [B] int64
    ctx_len: torch.Tensor      # [B] int32 (= position + 1)
    block_tables: torch.Tensor  # [B, max_blocks] int32
    count_row: torch.Tensor    # [B] int32 (sequence slot for penalty counts)
    temperature: torch.Tensor  # [B] f32
    penalty: torch.Tensor      # [B] f32
    top_k: torch.Tensor        # [B] int32
    top_p: torch.Tensor        # [B] f32
    tokens: torch.Tensor       # [B] int32 output
    probs: torch.Tensor        # [B] f32 output (top-1 prob of the filtered nucleus)
    mask: torch.Tensor         # [B, ceil(V/32)] int32 grammar allow-bits (all ones = no constraint)


class ModelRunner:
    def __init__(self, cfg: ModelConfig, weights: LlamaWeights, *, num_blocks: int,
                 block_size: int = 16, max_batch: int = 64, max_model_len: int = 4096,
                 max_seqs: int = 256, max_prefill_tokens: int = 8192, device="cuda", tp=None,
                 seed: int = 0, use_gemm_kernel: bool = True, kv_alloc=None, kv_dtype: str = "bf16"):
        """``kv_alloc(nbytes) -> uint8 CUDA tensor`` supplies the KV pool's memory (e.g. a
        cudaMalloc'd buffer exported over CUDA IPC for prefill->decode KV pushes).
        ``kv_dtype``: "bf16" pool rows of head_dim values, or "fp8": uint8 rows of head_dim
        E4M3 codes + f32 scale + padding (written by the RoPE/KV kernel, read by every
        attention kernel; reference: the Q8_0 KV option of src/kv_cache.rs:54-92)."""
        self.cfg, self.w = cfg, weights
        self.device = torch.device(device)
        self.tp = tp
        tp_size = tp.world_size if tp is not None else 1
        self.tp_size = tp_size
        self.nh = cfg.n_heads // tp_size
        self.nkv = max(1, cfg.n_kv_heads // tp_size)
        self.hd = cfg.head_dim
        self.H = cfg.hidden_dim
        # MoE experts are not split across TP ranks (expert parallelism places whole experts)
        self.F = cfg.intermediate_dim if cfg.n_experts else cfg.intermediate_dim // tp_size
        self.Fp = ops.pad32(self.F)  # activation width of the down projection (zero padded)
        self.V = cfg.vocab_size
        self.V_l = weights.lm_head.N
        self.block_size = block_size
        self.max_batch = max_batch
        self.max_model_len = max_model_len
        self.max_blocks = (max_model_len + block_size - 1) // block_size
        self.num_blocks = num_blocks
        self.seed = seed
        self.use_gemm_kernel = use_gemm_kernel
        dev = self.device
        L = len(weights.layers)          # this pipeline stage's layers
        from .builder import kv_row_bytes
        self.kv_dtype = kv_dtype
        self.kv_fp8 = kv_dtype == "fp8"
        row_b = kv_row_bytes(self.hd, kv_dtype)
        if self.kv_fp8 and self.hd % 64:
            raise ValueError("fp8 KV needs head_dim a multiple of 64")
        kv_t = torch.uint8 if self.kv_fp8 else torch.bfloat16
        esz = 1 if self.kv_fp8 else 2
        kv_shape = (L, num_blocks, 2, self.nkv, block_size, row_b // esz)
        if kv_alloc is None:
            self.kv = torch.zeros(kv_shape, dtype=kv_t, device=dev)
        else:
            n = 1
            for d_ in kv_shape:
                n *= d_
            self._kv_buf = kv_alloc(esz * n)
            self.kv = self._kv_buf[: esz * n].view(kv_t).view(kv_shape)
        rot = self.hd if cfg.partial_rope_factor is None else int(self.hd * cfg.partial_rope_factor)
        self.rot_dim = rot
        self.rope_cs = ops.rope_table(max_model_len + 64, rot, cfg.rope_theta, dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        self.counts = torch.zeros(max_seqs, self.V, dtype=torch.uint8, device=dev)
        self.step_ctr = torch.zeros(1, dtype=torch.int64, device=dev)
        self.qkv_dim = (self.nh + 2 * self.nkv) * self.hd
        from ..models.archs.hybrid import layout_for_config
        l0 = getattr(weights, "layer_range", (0, cfg.n_layers))[0]
        # per-layer attention window (0 = whole context): sliding / global interleaving
        self.layer_window = layout_for_config(cfg).windows()[l0:l0 + len(weights.layers)]
        B = max_batch
        kmax = max(self.H, self.Fp, self.nh * self.hd)
        f32, i8, bf16 = torch.float32, torch.int8, torch.bfloat16
        # decode workspace (sized for max_batch; buckets use leading slices)
        self.x = torch.zeros(B, self.H, dtype=f32, device=dev)
        self.xq = torch.zeros(B, kmax, dtype=i8, device=dev)
        self.xds = torch.zeros(B, kmax // 32, 2, dtype=f32, device=dev)
        self.q = torch.zeros(B, self.nh, self.hd, dtype=f32, device=dev)
        self.attn = torch.zeros(B, self.nh * self.hd, dtype=f32, device=dev)
        self.h = torch.zeros(B, self.Fp, dtype=f32, device=dev)
        gb = min(B, GEMV_LIMIT_B)
        self.gemv_max_b = GEMV_MAX_B
        self.hq = torch.zeros(gb, self.Fp, dtype=i8, device=dev)          # SwiGLU output, Q8A
        self.hds = torch.zeros(gb, self.Fp // 32, 2, dtype=f32, device=dev)
        # fused-norm decode chain: attention output (Q8A) and per-32-row sums of squares
        self.aq = torch.zeros(gb, self.nh * self.hd, dtype=i8, device=dev)
        self.ads = torch.zeros(gb, self.nh * self.hd // 32, 2, dtype=f32, device=dev)
        self.ss = torch.zeros(gb, self.H // 32, dtype=f32, device=dev)
        self.y = torch.zeros(B, self.H, dtype=f32, device=dev)
        self.logits = torch.zeros(B, self.V_l, dtype=f32, device=dev)
        self.logits_full = self.logits if tp_size == 1 else torch.zeros(B, self.V, dtype=f32, device=dev)
        # greedy steps under TP: per-rank partial argmax pass, all-gather of the partials
        # ([W, B, chunks] float4) instead of the [B, V] logits, device merge
        self.vocab_greedy = (tp_size > 1 and self.V_l < self.V and self.V_l % 32 == 0 and
                             os.environ.get("AIR_VOCAB_GREEDY", "0") == "1")
        self.head_greedy = False          # set per step by decode(greedy=...)
        if self.vocab_greedy:
            self.vnch = ops.sampler_chunks(self.V_l)
            self.vpart = torch.zeros(B * self.vnch * 4, dtype=f32, device=dev)
            self.vpart_all = torch.zeros(tp_size * B * self.vnch * 4, dtype=f32, device=dev)
        self.max_splits = 32
        self.part_o = torch.zeros(B * self.nh * self.max_splits * self.hd, dtype=f32, device=dev)
        self.part_ml = torch.zeros(B * self.nh * self.max_splits * 2, dtype=f32, device=dev)
        # GEMM-path activations (bf16) for large-batch decode
        self.xn_b = torch.zeros(B, self.H, dtype=bf16, device=dev)
        self.qkv_b = torch.zeros(B, self.qkv_dim, dtype=bf16, device=dev)
        self.attn_b = torch.zeros(B, self.nh * self.hd, dtype=bf16, device=dev)
        l0 = weights.layers[0]
        # architecture variant (reference src/model.rs:400-416, :623-660): norm kind, gate
        # activation, dense (ungated) MLP, q/k/v biases
        from ..models.config import FfnType, NormType
        self.norm_layer = cfg.norm_type == NormType.LAYER
        self.norm_off = 1.0 if cfg.norm_type == NormType.GEMMA_RMS else 0.0
        self.act = ops.ACT_GELU if cfg.ffn_type in (FfnType.GEGLU, FfnType.DENSE) else ops.ACT_SILU
        self.dense_ffn = cfg.ffn_type == FfnType.DENSE and not cfg.n_experts
        self.qkv_bias = l0.qkv_bias is not None
        self.gu_w = l0.wgu.N if l0.wgu is not None else 2 * self.F   # gate|up GEMM width
        if self.dense_ffn:
            self.up_off = -1           # the "gate|up" GEMM output is the up projection alone
        else:
            self.up_off = l0.wgu.parts[1][0] if l0.wgu is not None else self.F
        self.qkv_f = (torch.zeros(B, self.qkv_dim, dtype=f32, device=dev)
                      if self.qkv_bias or self.kv_fp8 else None)
        # decode GEMVs read Q4_K / Q8_0 / bf16; other formats (block-scaled FP8) decode on the
        # tensor-core GEMM path at every batch size
        fmts = [q.fmt for lw in weights.layers for q in (lw.wqkv, lw.wo, lw.wgu, lw.wdown) if q is not None]
        fmts += [q.fmt for lw in weights.layers for q in lw.experts_gu + lw.experts_down] + [weights.lm_head.fmt]
        self.gemv_ok = all(f in ops.GEMV_FMTS for f in fmts)
        self.gu_b = torch.zeros(B, self.gu_w, dtype=bf16, device=dev)
        self.h_b = torch.zeros(B, self.Fp, dtype=bf16, device=dev)
        self.o_b = torch.zeros(B, self.H, dtype=bf16, device=dev)
        self.inputs: dict[int, StepInputs] = {}
        # keyed by (bucket, greedy head): greedy steps under TP capture the partial-merge head
        self.graphs: dict[tuple, torch.cuda.CUDAGraph] = {}
        self.graph_launches: dict[tuple, int] = {}
        self.graph_comm: dict[tuple, dict] = {}      # collective calls / bytes per replay
        self._prefill_ws: dict[str, torch.Tensor] = {}
        self.streamer = None
        self.expert_cache = None
        self.max_prefill_tokens = max_prefill_tokens
        self._wscratch = None

    # ------------------------------------------------------------------ layer weights
    def _layer(self, li: int):
        """Layer li's weights on the device (resident, or streamed into a slot)."""
        if self.streamer is not None:
            return self.streamer.get(li)
        return self.w.layers[li]

    def _layer_done(self, li: int):
        if self.streamer is not None:
            self.streamer.release(li)

    def enable_expert_cache(self, capacity: int):
        """Serve host-resident MoE experts through ``capacity`` device slots (LRU)."""
        from .expert_cache import DeviceExpertCache
        if not any(lw.experts_gu for lw in self.w.layers):
            raise ValueError("expert cache needs a MoE model")
        self.expert_cache = DeviceExpertCache(self.w.layers, capacity, self.device)
        self.graphs.clear()
        return self.expert_cache

    def enable_streaming(self, n_slots: int = 2, resident_layers: int = 0):
        """Stream host-resident layers through ``n_slots`` device slots (S.L.I.P.); the first
        ``resident_layers`` layers are copied to the device once and stay there."""
        from ..stream.slip import LayerStreamer
        self.streamer = LayerStreamer(self.w.layers, self.device, n_slots, resident=range(resident_layers))
        return self.streamer

    # ------------------------------------------------------------------ inputs
    def step_inputs(self, B: int) -> StepInputs:
        si = self.inputs.get(B)
        if si is None:
            d = self.device
            si = StepInputs(
                ids=torch.zeros(B, dtype=torch.int32, device=d),
                positions=torch.zeros(B, dtype=torch.int32, device=d),
                slots=torch.full((B,), -1, dtype=torch.int64, device=d),
                ctx_len=torch.ones(B, dtype=torch.int32, device=d),
                block_tables=torch.full((B, self.max_blocks), -1, dtype=torch.int32, device=d),
                count_row=torch.arange(B, dtype=torch.int32, device=d),
                temperature=torch.zeros(B, dtype=torch.float32, device=d),
                penalty=torch.ones(B, dtype=torch.float32, device=d),
                top_k=torch.zeros(B, dtype=torch.int32, device=d),
                top_p=torch.ones(B, dtype=torch.float32, device=d),
                tokens=torch.zeros(B, dtype=torch.int32, device=d),
                probs=torch.zeros(B, dtype=torch.float32, device=d),
                mask=torch.full((B, (self.V + 31) // 32), -1, dtype=torch.int32, device=d),
            )
            self.inputs[B] = si
        return si

    def n_splits(self, B: int) -> int:
        target = 4 * 148
        return int(max(1, min(self.max_splits, math.ceil(target / max(1, B * self.nkv)))))

    # ------------------------------------------------------------------ linear (GEMM path)
    def linear(self, x_bf16: torch.Tensor, w: ops.QWeight, out: torch.Tensor,
               residual: bool = False) -> torch.Tensor:
        """out[T, N] = x[T, K] @ W^T (out += ... when residual) for the GEMM path."""
        from ..ops import gemm
        return gemm.linear(x_bf16, w, out, self, residual=residual, err=self.err)

    def linear_rows(self, x_bf16, w: ops.QWeight, out, row_count: torch.Tensor):
        """``linear`` for the first ``row_count`` (device int32) rows; later rows are left
        unspecified (routed-expert groups launched for a fixed capacity)."""
        from ..ops import gemm
        if gemm.tc_supported(w):
            return gemm.linear(x_bf16, w, out, self, err=self.err, row_count=row_count)
        return gemm.linear(x_bf16, w, out, self, err=self.err)

    def _proj_into_residual(self, xin, w, x, obuf, tp: bool, peer=None):
        """x += xin @ W^T: fused into the GEMM epilogue, or partial + all-reduce under TP.

        With a peer communicator the partial is pushed to every rank instead and the sum
        happens in the next ``_norm`` (decode only)."""
        T = xin.shape[0]
        if peer is not None:
            from ..ops import gemm
            if gemm.tc_supported(w):
                peer.push_gemm(xin, w, self.y[:T], err=self.err)   # push from the GEMM epilogue
            else:
                self.linear(xin, w, self.y[:T])
                peer.push(self.y[:T], T)
        elif tp:
            self.linear(xin, w, obuf[:T])
            self._residual_T(obuf[:T], T, x, tp)
        else:
            self.linear(xin, w, x, residual=True)

    # ------------------------------------------------------------------ collectives
    def _reduce_into_residual(self, partial: torch.Tensor, B: int, x: torch.Tensor):
        """x += all_reduce(partial) across TP ranks (partial: [B, H] f32)."""
        self.tp.all_reduce_add(partial[:B], x[:B])

    def _peer(self, B: int):
        """The fused peer-memory all-reduce for a decode batch of B rows, if any."""
        peer = getattr(self.tp, "peer", None) if self.tp_size > 1 else None
        return peer if peer is not None and peer.fits(B, self.H) else None

    def _row_parallel(self, w, xq, xds, B: int, x, peer):
        """Decode GEMV of a row-parallel projection: x += sum over ranks of xq @ W^T."""
        if peer is not None:
            if w.fmt == ops.FMT_Q4K:
                peer.push_gemv(w, xq, xds, B, err=self.err)
            else:
                ops.gemv(w, xq, xds, B, ops.EPI_STORE, out_f32=self.y[:B])
                peer.push(self.y[:B], B)
        elif self.tp_size > 1:
            ops.gemv(w, xq, xds, B, ops.EPI_STORE, out_f32=self.y[:B])
            self._reduce_into_residual(self.y, B, x)
        else:
            ops.gemv(w, xq, xds, B, ops.EPI_RESIDUAL, resid=x)

    def _norm(self, x, w, B: int, xq=None, xds=None, y_bf16=None, peer=None, bias=None):
        """The architecture's norm (+quant) of the residual stream; first completes a pending
        peer reduce."""
        eps = self.cfg.rms_norm_eps
        if peer is not None and peer.pending:
            peer.reduce_norm(x[:B], w, eps, xq, xds, y_bf16, B, w_offset=self.norm_off, bias=bias,
                             layer=self.norm_layer)
        else:
            ops.rmsnorm_quant(x[:B], w, eps, xq, xds, y_bf16=y_bf16, w_offset=self.norm_off, bias=bias,
                              layer=self.norm_layer)

    def _qkv_gemm_rope(self, xin, lw, qkv_buf, positions, slots, kv, q_out):
        """QKV projection on the GEMM path, then RoPE + paged KV write (token-parallel kernel;
        folding it into the GEMM epilogue measured slower, the epilogue is serial after the
        main loop while this kernel overlaps the next launch under PDL)."""
        T = xin.shape[0]
        self.linear(xin, lw.wqkv, qkv_buf)
        ops.rope_kv(qkv_buf, T, self.rope_cs, positions, slots, kv, q_out, n_heads=self.nh, n_kv=self.nkv,
                    head_dim=self.hd, block_size=self.block_size, rot_dim=self.rot_dim, err=self.err,
                    bias=lw.qkv_bias)

    def _qkv_rope(self, lw, xq, xds, B, kv, si):
        """Decode QKV GEMV + RoPE + paged KV write (fused epilogue; with q/k/v biases the
        GEMV stores and the token-parallel RoPE kernel adds the bias first)."""
        if self.qkv_f is not None:
            # q/k/v biases, or an fp8 pool (the per-row E4M3 scale needs the whole head row)
            ops.gemv(lw.wqkv, xq, xds, B, ops.EPI_STORE, out_f32=self.qkv_f[:B])
            ops.rope_kv(self.qkv_f[:B], B, self.rope_cs, si.positions, si.slots, kv, self.q[:B],
                        n_heads=self.nh, n_kv=self.nkv, head_dim=self.hd, block_size=self.block_size,
                        rot_dim=self.rot_dim, err=self.err, bias=lw.qkv_bias)
            return
        ops.gemv(lw.wqkv, xq, xds, B, ops.EPI_QKV_ROPE, rope_cs=self.rope_cs,
                 positions=si.positions, slots=si.slots, kv=kv, q_out=self.q[:B],
                 n_heads=self.nh, n_kv=self.nkv, head_dim=self.hd,
                 block_size=self.block_size, rot_dim=self.rot_dim, err=self.err)

    # ------------------------------------------------------------------ decode
    def _decode_body(self, B: int):
        if B <= self.gemv_max_b and self.gemv_ok and self.fused_norm_ok():
            return self._decode_fused(B)
        cfg, w, si = self.cfg, self.w, self.inputs[B]
        x, xq, xds = self.x[:B], self.xq[:B], self.xds[:B]
        ops.embed(w.embd, si.ids, out_f32=x, err=self.err, n=B)
        gemv_path = B <= self.gemv_max_b and self.gemv_ok
        ns = self.n_splits(B)
        tp = self.tp_size > 1
        peer = self._peer(B)
        for li in range(len(w.layers)):
            lw = self._layer(li)
            kv = self.kv[li]
            if gemv_path:
                self._norm(x, lw.attn_norm, B, xq, xds, peer=peer, bias=lw.attn_norm_b)
                self._qkv_rope(lw, xq, xds, B, kv, si)
            else:
                self._norm(x, lw.attn_norm, B, y_bf16=self.xn_b[:B], peer=peer, bias=lw.attn_norm_b)
                self._qkv_gemm_rope(self.xn_b[:B], lw, self.qkv_b[:B], si.positions, si.slots, kv, self.q[:B])
            ops.paged_attention(self.q[:B], kv, si.block_tables, si.ctx_len, self.attn[:B],
                                n_rows=B, n_heads=self.nh, n_kv=self.nkv, head_dim=self.hd,
                                block_size=self.block_size, n_splits=ns if gemv_path else max(2, ns),
                                split_tokens=0, part_o=self.part_o, part_ml=self.part_ml,
                                out_q=xq if gemv_path else None, out_ds=xds if gemv_path else None,
                                err=self.err, window=self.layer_window[li], softcap=cfg.attn_softcap,
                                out_bf16=None if gemv_path else self.attn_b[:B])
            if gemv_path:
                self._row_parallel(lw.wo, xq, xds, B, x, peer)
                # MoE layers also need the bf16 normalised row for the router
                self._norm(x, lw.ffn_norm, B, xq, xds, y_bf16=self.xn_b[:B] if lw.wgu is None else None, peer=peer,
                           bias=lw.ffn_norm_b)
                self._ffn_gemv(lw, B, x, xq, xds, tp, peer)
            else:
                self._proj_into_residual(self.attn_b[:B], lw.wo, x, self.o_b, tp, peer)
                self._norm(x, lw.ffn_norm, B, y_bf16=self.xn_b[:B], peer=peer, bias=lw.ffn_norm_b)
                self._ffn_gemm(lw, B, x, tp, peer)
            self._layer_done(li)
        self._head(B, x, xq, xds, gemv_path, peer)

    def fused_norm_ok(self) -> bool:
        """Decode GEMV chain with the RMSNorms folded into the GEMV epilogues: one GPU, dense
        layers, every projection in the tiled Q4_K layout, resident weights."""
        if getattr(self, "_fused_ok", None) is None:
            q4 = lambda q: q is not None and q.fmt == ops.FMT_Q4K
            w = self.w
            self._fused_ok = (self.tp_size == 1 and self.hd == 128 and q4(w.lm_head) and
                              os.environ.get("AIR_FUSED_NORM", "1") != "0" and
                              not self.norm_layer and not self.dense_ffn and not self.qkv_bias and
                              not self.kv_fp8 and
                              all(lw.wgu is not None and q4(lw.wqkv) and q4(lw.wo) and q4(lw.w_gate) and
                                  q4(lw.wdown) for lw in w.layers))
        return self._fused_ok and self.streamer is None

    def _decode_fused(self, B: int):
        """B <= 8 decode where each residual GEMV (o, down) also emits the next RMSNorm's
        quantised input and row sums of squares, and the next GEMV applies the 1/rms scale in
        its epilogue: one norm kernel per step (the first) instead of two per layer."""
        cfg, w, si = self.cfg, self.w, self.inputs[B]
        H, eps = self.H, cfg.rms_norm_eps
        x = self.x[:B]
        xa = self.xq.view(-1)[: B * H].view(B, H)
        xda = self.xds.view(-1)[: B * H // 16].view(B, H // 32, 2)
        aq, ads, hq, hds = self.aq[:B], self.ads[:B], self.hq[:B], self.hds[:B]
        # one partial-sum buffer suffices: every GEMV writes it only after griddepcontrol.wait,
        # i.e. after the previous consumer has finished reading it
        ss = self.ss[:B]
        ops.embed(w.embd, si.ids, out_f32=x, err=self.err, n=B)
        ops.rmsnorm_quant(x, w.layers[0].attn_norm, eps, xa, xda, w_offset=self.norm_off)
        ns = self.n_splits(B)
        L = len(w.layers)
        for li in range(L):
            lw = w.layers[li]
            kv = self.kv[li]
            ops.gemv(lw.wqkv, xa, xda, B, ops.EPI_QKV_ROPE, rope_cs=self.rope_cs,
                     positions=si.positions, slots=si.slots, kv=kv, q_out=self.q[:B],
                     n_heads=self.nh, n_kv=self.nkv, head_dim=self.hd,
                     block_size=self.block_size, rot_dim=self.rot_dim, err=self.err,
                     ss_in=ss if li > 0 else None, norm_k=H, eps=eps)
            ops.paged_attention(self.q[:B], kv, si.block_tables, si.ctx_len, self.attn[:B],
                                n_rows=B, n_heads=self.nh, n_kv=self.nkv, head_dim=self.hd,
                                block_size=self.block_size, n_splits=ns, split_tokens=0,
                                part_o=self.part_o, part_ml=self.part_ml, out_q=aq, out_ds=ads,
                                err=self.err, window=self.layer_window[li], softcap=cfg.attn_softcap)
            ops.gemv(lw.wo, aq, ads, B, ops.EPI_RESIDUAL, resid=x, norm_w=lw.ffn_norm, out_q=xa, out_ds=xda,
                     ss_out=ss, norm_offset=self.norm_off)
            ops.gemv(lw.w_gate, xa, xda, B, ops.EPI_SWIGLU, w2=lw.w_up, ld_out=self.Fp, out_q=hq, out_ds=hds,
                     ss_in=ss, norm_k=H, eps=eps, act=self.act)
            nxt = w.layers[li + 1].attn_norm if li + 1 < L else w.out_norm
            ops.gemv(lw.wdown, hq, hds, B, ops.EPI_RESIDUAL, resid=x, norm_w=nxt, out_q=xa, out_ds=xda,
                     ss_out=ss, norm_offset=self.norm_off)
        ops.gemv(w.lm_head, xa, xda, B, ops.EPI_STORE, out_f32=self.logits[:B], ss_in=ss, norm_k=H, eps=eps)
        ops.sample(self.logits[:B], si.tokens, counts=self.counts, count_row=si.count_row, mask=si.mask,
                   temperature=si.temperature, penalty=si.penalty, top_k=si.top_k, top_p=si.top_p,
                   seed=self.seed, step=self.step_ctr, out_prob=si.probs, B=B, V=self.V)
        ops.count_tokens(self.counts, si.tokens, n=B, count_row=si.count_row)
        si.ids.copy_(si.tokens)

    def _residual(self, y_b: torch.Tensor, B: int, x: torch.Tensor, tp: bool):
        if tp:
            self.y[:B].copy_(y_b[:B])
            self._reduce_into_residual(self.y, B, x)
        else:
            ops.residual_add(x, y_b[:B])

    def _ffn_gemv(self, lw, B, x, xq, xds, tp, peer=None):
        if lw.wgu is None:
            from ..parallel import moe
            moe.moe_ffn_decode(self, lw, B, x, xq, xds, peer)
            return
        if self.dense_ffn:
            # dense GELU MLP: up GEMV, GELU, quantise, down
            ops.gemv(lw.wgu, xq, xds, B, ops.EPI_STORE, out_f32=self.h[:B], ld_out=self.Fp)
            ops.swiglu(self.h[:B], B, self.F, out_f32=self.h[:B], ld_out=self.Fp, up_off=-1, act=self.act)
            ops.rmsnorm_quant(self.h[:B], None, 0.0, xq, xds)
            self._row_parallel(lw.wdown, xq, xds, B, x, peer)
            return
        if lw.w_gate.fmt == ops.FMT_Q4K:
            # gated product quantised in the GEMV epilogue (no separate quant kernel)
            hq, hds = self.hq[:B], self.hds[:B]
            ops.gemv(lw.w_gate, xq, xds, B, ops.EPI_SWIGLU, w2=lw.w_up, ld_out=self.Fp, out_q=hq, out_ds=hds,
                     act=self.act)
            self._row_parallel(lw.wdown, hq, hds, B, x, peer)
            return
        ops.gemv(lw.w_gate, xq, xds, B, ops.EPI_SWIGLU, w2=lw.w_up, out_f32=self.h[:B], ld_out=self.Fp,
                 act=self.act)
        ops.rmsnorm_quant(self.h[:B], None, 0.0, xq, xds)
        self._row_parallel(lw.wdown, xq, xds, B, x, peer)

    def _ffn_gemm(self, lw, B, x, tp, peer=None):
        if lw.wgu is None:
            from ..parallel import moe
            moe.moe_ffn_gemm(self, lw, B, x, peer)
            return
        self.linear(self.xn_b[:B], lw.wgu, self.gu_b[:B])
        ops.swiglu(self.gu_b[:B], B, self.F, out_bf16=self.h_b[:B], ld_out=self.Fp, up_off=self.up_off,
                   act=self.act)
        self._proj_into_residual(self.h_b[:B], lw.wdown, x, self.o_b, tp, peer)

    def _head(self, B, x, xq, xds, gemv_path, peer=None):
        w, si = self.w, self.inputs[B]
        if gemv_path:
            self._norm(x, w.out_norm, B, xq, xds, peer=peer, bias=w.out_norm_b)
            ops.gemv(w.lm_head, xq, xds, B, ops.EPI_STORE, out_f32=self.logits[:B])
        else:
            self._norm(x, w.out_norm, B, y_bf16=self.xn_b[:B], peer=peer, bias=w.out_norm_b)
            self.linear(self.xn_b[:B], w.lm_head, self.logits[:B])
        logits = self.logits[:B]
        if self.tp_size > 1 and self.head_greedy and self.vocab_greedy:
            self._head_greedy_tp(B, si)
            return
        if self.tp_size > 1:
            logits = self.tp.all_gather_vocab(self.logits[:B], self.logits_full[:B])
        ops.sample(logits, si.tokens, counts=self.counts, count_row=si.count_row, mask=si.mask,
                   temperature=si.temperature, penalty=si.penalty, top_k=si.top_k, top_p=si.top_p,
                   seed=self.seed, step=self.step_ctr, out_prob=si.probs, B=B, V=self.V)
        ops.count_tokens(self.counts, si.tokens, n=B, count_row=si.count_row)
        si.ids.copy_(si.tokens)

    def _head_greedy_tp(self, B: int, si: StepInputs):
        """Vocabulary-parallel greedy sampling: this rank's penalised, masked argmax per
        1024-column chunk of its logit shard, one all-gather of [B, chunks] float4 partials
        (B x 126 x 16 bytes per rank at V = 128K, TP 8; the logits are B x 64 KB), and the
        argmax merge on every rank. Same tokens as the whole-vocabulary sampler at
        temperature 0 (lowest index on ties). Reference: the sampler's greedy branch
        (src/sampler.rs:83-120) over logits gathered to one device."""
        W, r, nch = self.tp_size, self.tp.rank, self.vnch
        v_off = r * self.V_l
        valid = max(0, min(self.V_l, self.V - v_off))
        part = self.vpart[:B * nch * 4]
        ops.sample_partial(self.logits[:B], part, v_off=v_off, V_total=self.V, counts=self.counts,
                           count_row=si.count_row, mask=si.mask, penalty=si.penalty, B=B, V=valid, nch=nch)
        allp = self.vpart_all[:W * B * nch * 4]
        self.tp.all_gather_flat(part, allp)
        ops.sample_greedy_merge(allp, si.tokens, W=W, B=B, nch=nch, out_prob=si.probs, step=self.step_ctr)
        ops.count_tokens(self.counts, si.tokens, n=B, count_row=si.count_row)
        si.ids.copy_(si.tokens)

    def decode(self, B: int, use_graph: bool = True, greedy: bool = False):
        """Runs one decode step for the first B rows of the bucket-B inputs. ``greedy``: every
        row samples at temperature 0 (lets a TP step merge per-rank argmax partials instead
        of gathering the logits)."""
        self.step_inputs(B)
        self.head_greedy = bool(greedy) and self.vocab_greedy
        if not use_graph or self.streamer is not None or self.expert_cache is not None:
            self._decode_body(B)
            return self.inputs[B]
        key = (B, self.head_greedy)
        g = self.graphs.get(key)
        if g is None:
            # The warm-up run (lazy init outside capture) mutates step state: sampled ids,
            # penalty counts, the Philox step counter. Snapshot and restore it so the first
            # real step sees exactly the inputs the host staged.
            si = self.inputs[B]
            saved = (si.ids.clone(), self.counts.clone(), self.step_ctr.clone())
            s = torch.cuda.Stream(self.device)
            s.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(s):
                self._decode_body(B)
            torch.cuda.current_stream(self.device).wait_stream(s)
            si.ids.copy_(saved[0])
            self.counts.copy_(saved[1])
            self.step_ctr.copy_(saved[2])
            del saved
            g = torch.cuda.CUDAGraph()
            c0 = ops.launch_count()
            m0 = COMM.snapshot()
            # capture on a stream of this runner's device: torch.cuda.graph's default capture
            # stream is created once per process on whichever device was current then, and
            # entering it switches the current device, so a second GPU in the same process
            # (an in-process prefill/decode pair) would record its kernels on the first GPU
            if getattr(self, "_capture_stream", None) is None:
                self._capture_stream = torch.cuda.Stream(self.device)
            with torch.cuda.graph(g, stream=self._capture_stream):
                self._decode_body(B)
            self.graph_launches[key] = ops.launch_count() - c0
            ops.count_launch(-(ops.launch_count() - c0))  # capture itself runs nothing
            self.graph_comm[key] = COMM.since(m0)
            COMM.add(self.graph_comm[key], sign=-1)
            self.graphs[key] = g
        g.replay()
        ops.count_launch(self.graph_launches[key])
        COMM.add(self.graph_comm[key])
        return self.inputs[B]

    # ------------------------------------------------------------------ prefill
    def _ws(self, name, shape, dtype, zero: bool = False):
        t = self._prefill_ws.get(name)
        n = 1
        for s in shape:
            n *= s
        if t is None or t.numel() < n or t.dtype != dtype:
            t = (torch.zeros if zero else torch.empty)(max(n, 1), dtype=dtype, device=self.device)
            self._prefill_ws[name] = t
        return t[:n].view(*shape)

    def prefill(self, ids: torch.Tensor, positions: torch.Tensor, slots: torch.Tensor,
                row_seq: torch.Tensor, block_tables: torch.Tensor, last_rows: torch.Tensor,
                count_rows: torch.Tensor, temperature, penalty, top_k, top_p, mask=None,
                return_hidden: bool = False, tree_base: torch.Tensor | None = None,
                tree_mask: torch.Tensor | None = None, return_logits: bool = False,
                ctx_len: torch.Tensor | None = None, hidden_in: torch.Tensor | None = None,
                return_hidden_out: bool = False, return_final_hidden: bool = False):
        """Prompt tokens of one or more sequences (concatenated, T total).

        row_seq[t] indexes ``block_tables``; last_rows[s] is the row of each sequence's last
        token, whose logits are sampled. Returns (tokens [S] int32, probs [S] f32).
        Pipeline stages: ``hidden_in`` [T, H] fp32 replaces the embedding (the previous
        stage's residual stream) and ``return_hidden_out`` returns the residual stream after
        this runner's layers instead of sampling.
        """
        cfg, w = self.cfg, self.w
        T = ids.numel()
        S = last_rows.numel()
        eps = cfg.rms_norm_eps
        f32, bf16 = torch.float32, torch.bfloat16
        x = self._ws("x", (T, self.H), f32)
        xn = self._ws("xn", (T, self.H), bf16)
        qkv = self._ws("qkv", (T, self.qkv_dim), bf16)
        q = self._ws("q", (T, self.nh, self.hd), f32)
        attn = self._ws("attn", (T, self.nh * self.hd), f32)
        attn_b = self._ws("attn_b", (T, self.nh * self.hd), bf16)
        o = self._ws("o", (T, self.H), bf16)
        gu = self._ws("gu", (T, self.gu_w), bf16) if self.w.layers[0].wgu is not None else None
        hb = self._ws("hb", (T, self.Fp), bf16, zero=True)
        # keys [0, ctx) are candidates; tree rows pass their own bound (slot-based, not position)
        ctx = ctx_len if ctx_len is not None else (positions + 1).to(torch.int32)
        tp = self.tp_size > 1
        if hidden_in is not None:
            x.copy_(hidden_in)
        else:
            ops.embed(w.embd, ids, out_f32=x, err=self.err, n=T)
        for li in range(len(w.layers)):
            _sp = trace.span(f"prefill/layer{li}") if trace.enabled() else None
            if _sp is not None:
                _sp.__enter__()
            lw = self._layer(li)
            kv = self.kv[li]
            ops.rmsnorm_quant(x, lw.attn_norm, eps, None, None, y_bf16=xn, bias=lw.attn_norm_b,
                              w_offset=self.norm_off, layer=self.norm_layer)
            self._qkv_gemm_rope(xn, lw, qkv, positions, slots, kv, q)
            ops.paged_attention(q, kv, block_tables, ctx, attn, n_rows=T, n_heads=self.nh,
                                n_kv=self.nkv, head_dim=self.hd, block_size=self.block_size,
                                row_seq=row_seq, n_splits=1, err=self.err,
                                window=self.layer_window[li], tree_base=tree_base, tree_mask=tree_mask,
                                softcap=cfg.attn_softcap)
            attn_b.copy_(attn)
            self._proj_into_residual(attn_b, lw.wo, x, o, tp)
            ops.rmsnorm_quant(x, lw.ffn_norm, eps, None, None, y_bf16=xn, bias=lw.ffn_norm_b,
                              w_offset=self.norm_off, layer=self.norm_layer)
            if lw.wgu is None:
                from ..parallel import moe
                moe.moe_ffn_prefill(self, lw, T, x, xn)
            else:
                self.linear(xn, lw.wgu, gu)
                ops.swiglu(gu, T, self.F, out_bf16=hb, ld_out=self.Fp, up_off=self.up_off, act=self.act)
                self._proj_into_residual(hb, lw.wdown, x, o, tp)
            self._layer_done(li)
            if _sp is not None:
                _sp.__exit__(None, None, None)
        if return_hidden_out:
            return x.clone()
        if return_hidden:  # final-norm hidden states of every row (embeddings)
            hn = self._ws("hn", (T, self.H), bf16)
            ops.rmsnorm_quant(x, w.out_norm, eps, None, None, y_bf16=hn, bias=w.out_norm_b,
                              w_offset=self.norm_off, layer=self.norm_layer)
            return hn.float()
        xl = x.index_select(0, last_rows.long())
        xs = self._ws("xs", (S, self.H), bf16)
        ops.rmsnorm_quant(xl, w.out_norm, eps, None, None, y_bf16=xs, bias=w.out_norm_b,
                          w_offset=self.norm_off, layer=self.norm_layer)
        logits = self._ws("logits", (S, self.V_l), f32)
        self.linear(xs, w.lm_head, logits)
        if tp:
            full = self._ws("logits_full", (S, self.V), f32)
            logits = self.tp.all_gather_vocab(logits, full)
        if return_logits:
            if return_final_hidden:      # (logits, final-norm hidden) of the last rows
                return logits[:, : self.V].clone(), xs.float().clone()
            return logits[:, : self.V].clone()
        toks = torch.zeros(S, dtype=torch.int32, device=self.device)
        probs = torch.zeros(S, dtype=torch.float32, device=self.device)
        ops.sample(logits, toks, counts=self.counts, count_row=count_rows, mask=mask, temperature=temperature,
                   penalty=penalty, top_k=top_k, top_p=top_p, seed=self.seed, step=self.step_ctr,
                   out_prob=probs, B=S, V=self.V)
        ops.count_tokens(self.counts, toks, n=S, count_row=count_rows)
        return toks, probs

    def _residual_T(self, o, T, x, tp):
        if tp:
            y = self._ws("y", (T, self.H), torch.float32)
            y.copy_(o)
            self.tp.all_reduce_add(y, x)
        else:
            ops.residual_add(x, o)

    # ------------------------------------------------------------------ misc
    def embed_ids(self, ids: torch.Tensor) -> torch.Tensor:
        """Token embeddings [T, H] fp32 (the rows prefill starts from)."""
        out = torch.empty(ids.numel(), self.H, dtype=torch.float32, device=self.device)
        ops.embed(self.w.embd, ids, out_f32=out, err=self.err, n=ids.numel())
        return out

    def check_errors(self):
        peer = getattr(self.tp, "peer", None) if self.tp_size > 1 else None
        if peer is not None:
            peer.check()
        e = int(self.err.item())
        if e:
            self.err.zero_()
            raise RuntimeError(f"device kernel reported error code {e} (1=index out of range, 2=peer timeout)")

    def reset_counts(self, row: int, prompt_ids: torch.Tensor | None = None):
        self.counts[row].zero_()
        if prompt_ids is not None and prompt_ids.numel():
            cr = torch.full((prompt_ids.numel(),), row, dtype=torch.int32, device=self.device)
            ops.count_tokens(self.counts, prompt_ids.to(self.device, torch.int32), count_row=cr, per_row=1)
